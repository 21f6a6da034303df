"""Preallocated, current-stream binding of the fused residual prologue (B200).

x <- bf(fma(branch, bf(gate[rows]), x)) in place, then RMSNorm -> adaLN
x*(1+scale)+shift -> ConvRot256 -> per-token INT8 of the updated rows, one pass.
Drop-in for h3_speedkit/ops/residual_quant.py of H3 SpeedKit: the same class and
function names, argument meaning, validation messages and error behaviour
(``validate`` at :57-112, ``ResidualQuant`` at :115-153, ``Bound`` at :156-171),
with the differences of ``ops.norm_quant``: K is taken from ``x`` (any
K % 256 == 0 up to 16384, reference: 5376 only) and the device must be a B200.

X is both an input and the in-place output; the bound object owns the Torch
tensors; rows are immutable after validation.  Returned q/q_scale are the
prequantised Linear input.
"""
from __future__ import annotations

import ctypes as ct
import math

import torch

from .. import _lib
from .norm_quant import DEVICE_CAPABILITY, K, MAX_K, Resources, check_disjoint, finite_bounded, span

__all__ = ["K", "Resources", "span", "check_disjoint", "finite_bounded", "validate", "ResidualQuant", "Bound"]


def validate(x, branch, weight, gate, shift, scale, rows, q, q_scale, *, eps,
             debug_norm=None, debug_rotated=None, debug_rstd=None,
             check_values=True, require_cuda=True):
    """Metadata checks; runnable on CPU tensors with require_cuda=False."""
    inputs = [('branch', branch), ('weight', weight), ('gate', gate), ('shift', shift), ('scale', scale),
              ('rows', rows)]
    outputs = [('x', x), ('q', q), ('q_scale', q_scale)]
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
        raise ValueError('X requires aligned contiguous BF16 [M,K]')
    m, k = x.shape
    if (k % 256 or not 256 <= k <= MAX_K or not 1 <= m <= 0x7fffffff or not x.is_contiguous()
            or x.data_ptr() % 8):
        raise ValueError(f'X requires aligned contiguous BF16 [M,{k}]')
    if (branch.shape != x.shape or branch.dtype != torch.bfloat16 or not branch.is_contiguous()
            or branch.data_ptr() % 8):
        raise ValueError(f'Branch requires aligned contiguous BF16 [M,{k}]')

    def dense(name, t, shape, dtype, alignment):
        if tuple(t.shape) != tuple(shape) or t.dtype != dtype or not t.is_contiguous() or t.data_ptr() % alignment:
            raise ValueError(f'{name} requires contiguous {dtype} {tuple(shape)} and {alignment}B alignment')

    dense('weight', weight, (k,), torch.bfloat16, 8)
    if (shift.ndim != 2 or shift.shape[1] != k or shift.shape[0] < 1 or shift.shape[0] > 0x7fffffff
            or scale.shape != shift.shape or shift.dtype != scale.dtype
            or shift.dtype not in (torch.bfloat16, torch.float32)):
        raise ValueError(f'Tables require matching nonempty FP32/BF16 [T,{k}]')
    if gate.shape != shift.shape or gate.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError('Gate requires matching table shape and independent FP32/BF16 dtype')
    for t in (gate, shift, scale):
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
        for tensor in (x, branch, weight, gate, shift, scale):
            finite_bounded(tensor)
    return tuple(inputs), tuple(outputs)


class ResidualQuant:
    """ctypes front of h3_residual_quant_* (libh3sk_b200.so)."""

    def __init__(self, library=None):
        self.lib = _lib.load(library)
        self.path = _lib.library_path() if library is None else library
        if self.lib.h3_residual_quant_abi() != 1 or \
                self.lib.h3_residual_quant_resources_size() != ct.sizeof(Resources):
            raise RuntimeError('ResidualQuant C/ctypes ABI mismatch')

    def check(self, code):
        if code:
            raise RuntimeError(f'ResidualQuant CUDA error {code}: ' + self.lib.h3_residual_quant_error(code).decode())

    def query(self, gate_dtype=0, table_dtype=0, debug=0, k=K):
        data = Resources()
        self.check(self.lib.h3_residual_quant_query_k(k, gate_dtype, table_dtype, debug, ct.byref(data),
                                                      ct.sizeof(data)))
        return {name: int(getattr(data, name)) for name, _ in data._fields_}

    def bind(self, x, branch, weight, gate, shift, scale, rows, q, q_scale, *, eps,
             debug_norm=None, debug_rotated=None, debug_rstd=None, check_values=True):
        inputs, outputs = validate(x, branch, weight, gate, shift, scale, rows, q, q_scale, eps=eps,
                                   debug_norm=debug_norm, debug_rotated=debug_rotated, debug_rstd=debug_rstd,
                                   check_values=check_values)
        with torch.cuda.device(x.device):
            if torch.cuda.get_device_capability(x.device) != DEVICE_CAPABILITY:
                raise RuntimeError('Only the intended B200 (sm_100) device is supported')
            if torch.compiler.is_compiling():
                raise RuntimeError('ResidualQuant requires eager execution')
        pointers = [t.data_ptr() for t in (x, branch, weight, gate, shift, scale, rows, q, q_scale)]
        pointers += [t.data_ptr() if t is not None else None for t in (debug_norm, debug_rotated, debug_rstd)]
        args = pointers + [x.shape[0], x.shape[1], shift.shape[0], gate.stride(0), shift.stride(0), scale.stride(0),
                           float(eps), int(gate.dtype == torch.bfloat16), int(shift.dtype == torch.bfloat16),
                           int(debug_norm is not None)]
        return Bound(self, x.device, inputs, outputs, args, (x, q, q_scale))


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
            code = self.library.lib.h3_residual_quant_run_t(*self.args, stream.cuda_stream)
            # Stores may already be queued when an error is reported: never retried.
            torch.autograd.graph.increment_version(tuple(t for _, t in self.outputs))
            self.library.check(code)
        return self.result
