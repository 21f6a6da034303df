"""Preallocated, current-stream binding of the fused residual prologue (B200).

x <- bf(fma(branch, bf(gate[rows]), x)) in place, then RMSNorm -> adaLN
x*(1+scale)+shift -> ConvRot256 -> per-token INT8 of the updated rows, one pass,
through ``h3_residual_quant_run_t``.  Stands in for
h3_speedkit/ops/residual_quant.py of H3 SpeedKit: the public names, argument
meaning and error texts are that module's (:57-171); the checks are a rule table
built from ``ops.norm_quant``'s (see ``_contract``), with the same two deliberate
differences: K is read off ``x`` (any K % 256 == 0 up to 16384; reference: 5376)
and the device must be a B200.

x is both an input and the in-place output.  Returned q / q_scale are the
prequantised Linear input.
"""
from __future__ import annotations

import ctypes as ct

import torch

from .. import _lib
from ._contract import INT32_MAX, Call, Launch, Rule, common_rules, debug_rule, dense_rule, disjoint_rule, enforce
from . import norm_quant as nq
from .norm_quant import (DEVICE_CAPABILITY, K, MAX_K, Resources, check_disjoint, finite_bounded,  # noqa: F401
                         require_device, span)

__all__ = ["K", "Resources", "span", "check_disjoint", "finite_bounded", "validate", "ResidualQuant", "Bound"]

INPUTS = ('branch', 'weight', 'gate', 'shift', 'scale', 'rows')
OUTPUTS = ('x', 'q', 'q_scale', 'debug_norm', 'debug_rotated', 'debug_rstd')


def _x_kind_ok(c):
    x = c['x']
    if x.dtype != torch.bfloat16 or x.ndim != 2:
        return False
    c.dims.update(m=x.shape[0], k=x.shape[1])
    return True


def _x_ok(c):
    x, (m, k) = c['x'], (c.dims['m'], c.dims['k'])
    return k % 256 == 0 and 256 <= k <= MAX_K and 1 <= m <= INT32_MAX and x.is_contiguous() and x.data_ptr() % 8 == 0


def _branch_ok(c):
    b, x = c['branch'], c['x']
    return b.shape == x.shape and b.dtype == torch.bfloat16 and b.is_contiguous() and b.data_ptr() % 8 == 0


RULES = [
    debug_rule(),
    *common_rules('x'),
    Rule(_x_kind_ok, 'X requires aligned contiguous BF16 [M,K]'),
    Rule(_x_ok, lambda c: f"X requires aligned contiguous BF16 [M,{c.dims['k']}]"),
    Rule(_branch_ok, lambda c: f"Branch requires aligned contiguous BF16 [M,{c.dims['k']}]"),
    dense_rule('weight', lambda c: (c.dims['k'],), torch.bfloat16, 8),
    Rule(lambda c: nq._tables_ok(c) and c['shift'].shape[0] <= INT32_MAX,
         lambda c: f"Tables require matching nonempty FP32/BF16 [T,{c.dims['k']}]"),
    Rule(lambda c: c['gate'].shape == c['shift'].shape and c['gate'].dtype in (torch.bfloat16, torch.float32),
         'Gate requires matching table shape and independent FP32/BF16 dtype'),
    Rule(lambda c: nq._table_rows_ok(c, ('gate', 'shift', 'scale')),
         'Tables require dense hidden axes and nonoverlapping rows'),
    dense_rule('rows', lambda c: (c.dims['m'],), torch.int32, 4),
    dense_rule('q', lambda c: (c.dims['m'], c.dims['k']), torch.int8, 8),
    dense_rule('q_scale', lambda c: (c.dims['m'], 1), torch.float32, 4),
    *nq._debug_rules(),
    Rule(lambda c: nq.normal_fp32(c.dims['eps']), 'Epsilon must be finite, positive, normal FP32'),
    disjoint_rule(INPUTS, OUTPUTS),
    *nq._value_rules('shift', ('x', 'branch', 'weight', 'gate', 'shift', 'scale')),
]


def validate(x, branch, weight, gate, shift, scale, rows, q, q_scale, *, eps,
             debug_norm=None, debug_rotated=None, debug_rstd=None,
             check_values=True, require_cuda=True):
    """Metadata checks (and, with check_values, the row-map and finiteness scans);
    runnable on CPU tensors with require_cuda=False."""
    names = {'x': x, 'branch': branch, 'weight': weight, 'gate': gate, 'shift': shift, 'scale': scale,
             'rows': rows, 'q': q, 'q_scale': q_scale, 'debug_norm': debug_norm,
             'debug_rotated': debug_rotated, 'debug_rstd': debug_rstd}
    enforce(RULES, Call(names, {'eps': eps, 'check_values': check_values, 'require_cuda': require_cuda}))
    return (tuple((n, names[n]) for n in INPUTS),
            tuple((n, names[n]) for n in OUTPUTS if names[n] is not None))


class ResidualQuant:
    """ctypes front of h3_residual_quant_* (libh3sk_b200.so)."""

    def __init__(self, library=None):
        self.lib = _lib.load(library)
        self.path = _lib.library_path() if library is None else library
        if (self.lib.h3_residual_quant_abi() != 1
                or self.lib.h3_residual_quant_resources_size() != ct.sizeof(Resources)):
            raise RuntimeError('ResidualQuant C/ctypes ABI mismatch')

    def check(self, code):
        if code:
            raise RuntimeError(f'ResidualQuant CUDA error {code}: ' + self.lib.h3_residual_quant_error(code).decode())

    def query(self, gate_dtype=0, table_dtype=0, debug=0, k=K):
        report = Resources()
        self.check(self.lib.h3_residual_quant_query_k(k, gate_dtype, table_dtype, debug, ct.byref(report),
                                                      ct.sizeof(report)))
        return {name: int(getattr(report, name)) for name, _ in report._fields_}

    def bind(self, x, branch, weight, gate, shift, scale, rows, q, q_scale, *, eps,
             debug_norm=None, debug_rotated=None, debug_rstd=None, check_values=True):
        inputs, outputs = validate(x, branch, weight, gate, shift, scale, rows, q, q_scale, eps=eps,
                                   debug_norm=debug_norm, debug_rotated=debug_rotated, debug_rstd=debug_rstd,
                                   check_values=check_values)
        require_device(x.device, 'ResidualQuant')
        ptr = lambda t: None if t is None else t.data_ptr()
        args = [ptr(t) for t in (x, branch, weight, gate, shift, scale, rows, q, q_scale, debug_norm, debug_rotated,
                                 debug_rstd)]
        args += [x.shape[0], x.shape[1], shift.shape[0], gate.stride(0), shift.stride(0), scale.stride(0),
                 float(eps), int(gate.dtype == torch.bfloat16), int(shift.dtype == torch.bfloat16),
                 int(debug_norm is not None)]
        return Bound(self.lib.h3_residual_quant_run_t, x.device, args, [t for _, t in inputs + outputs],
                     [t for _, t in outputs], (x, q, q_scale), self.check)


Bound = Launch
