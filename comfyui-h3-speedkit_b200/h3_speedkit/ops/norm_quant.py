"""Preallocated, current-stream binding of the fused prologue (B200).

RMSNorm -> adaLN x*(1+scale)+shift -> ConvRot256 -> per-token INT8, one pass,
through ``h3_norm_quant_run_t`` of libh3sk_b200.so.  Stands in for
h3_speedkit/ops/norm_quant.py of H3 SpeedKit: the public names (``validate``,
``NormQuant``, ``Bound``, ``Resources``, ``span``, ``check_disjoint``,
``finite_bounded``), the argument meaning and the error texts are that module's
(:57-164); the checks themselves are the rule table below (see ``_contract``).
Two deliberate differences: the hidden width K is read off ``x`` (any
K % 256 == 0 up to 16384; the reference accepts 5376 only) and the device must
be a B200 (capability 10.0; the reference requires SM120).

Returned q / q_scale are the prequantised Linear input.  Rows are immutable
after validation; callers order producers before bind and launch.
"""
from __future__ import annotations

import ctypes as ct

import torch

from .. import _lib
from ._contract import (INT32_MAX, Call, Launch, Rule, address_range, all_finite, common_rules, debug_rule,
                        dense_rule, disjoint_rule, enforce, first_overlap, normal_fp32)

K = 5376                      # width of the reference geometry (unsuffixed C entry point)
MAX_K = 16384
DEVICE_CAPABILITY = (10, 0)   # B200

INPUTS = ('x', 'weight', 'shift', 'scale', 'rows')
OUTPUTS = ('q', 'q_scale', 'debug_norm', 'debug_rotated', 'debug_rstd')
X_TEXT = 'X requires BF16 [M,K], unit columns, XS % 4 == 0, 8B alignment'


class Resources(ct.Structure):
    """h3_norm_quant_query's report (field order of norm_quant.cu:215-218)."""
    _fields_ = [(name, ct.c_int64) for name in (
        'abi', 'bytes', 'k', 'threads', 'warps', 'num_regs',
        'static_shared_bytes', 'local_bytes', 'active_blocks_per_sm',
        'sm_count', 'max_threads_per_sm', 'binary_version', 'ptx_version')]


def span(tensor):
    """Address interval [start, end) a strided tensor can touch."""
    return address_range(tensor)


def check_disjoint(inputs, outputs):
    """Outputs may overlap neither an input nor each other."""
    hit = first_overlap(list(inputs), list(outputs))
    if hit is not None:
        out, other, other_is_output = hit
        raise ValueError(f'Outputs {out} and {other} overlap' if other_is_output
                         else f'Output {out} overlaps input {other}')


def finite_bounded(tensor, rows=128):
    """Reject NaN/Inf, scanning 2-D tensors in bounded row chunks."""
    if not all_finite(tensor, rows):
        raise ValueError('Nonfinite input is outside the contract')


def _x_ok(c):
    x = c['x']
    if x.dtype != torch.bfloat16 or x.ndim != 2:
        return False
    m, k = x.shape
    c.dims.update(m=m, k=k)
    return (k % 256 == 0 and 256 <= k <= MAX_K and 1 <= m <= INT32_MAX and x.stride(1) == 1
            and x.stride(0) >= k and x.stride(0) % 4 == 0 and x.data_ptr() % 8 == 0)


def _tables_ok(c, names=('shift', 'scale')):
    k, first = c.dims['k'], c[names[0]]
    return (first.ndim == 2 and first.shape[1] == k and first.shape[0] >= 1
            and first.dtype in (torch.bfloat16, torch.float32)
            and all(c[n].shape == first.shape and c[n].dtype == first.dtype for n in names))


def _table_rows_ok(c, names=('shift', 'scale')):
    k = c.dims['k']
    return all(c[n].stride(1) == 1 and c[n].stride(0) >= k and c[n].data_ptr() % c[n].element_size() == 0
               for n in names)


def _debug_rules():
    mk = lambda c: (c.dims['m'], c.dims['k'])
    rules = [dense_rule('debug_norm', mk, torch.bfloat16, 2), dense_rule('debug_rotated', mk, torch.float32, 4),
             dense_rule('debug_rstd', lambda c: (c.dims['m'],), torch.float32, 4)]
    return [Rule(lambda c, r=r: c['debug_norm'] is None or r.ok(c), r.message) for r in rules]


def _value_rules(table, finite):
    """The value scans (optional: they synchronise with the device)."""
    return [
        Rule(lambda c: not c.dims['check_values'] or (int(c['rows'].min().item()) >= 0
                                                      and int(c['rows'].max().item()) < c[table].shape[0]),
             'Rows outside modulation table'),
        Rule(lambda c: not c.dims['check_values'] or all(all_finite(c[n]) for n in finite),
             'Nonfinite input is outside the contract'),
    ]


RULES = [
    debug_rule(),
    *common_rules('x'),
    Rule(_x_ok, X_TEXT),
    dense_rule('weight', lambda c: (c.dims['k'],), torch.bfloat16, 8),
    Rule(_tables_ok, lambda c: f"Tables require matching nonempty FP32/BF16 [T,{c.dims['k']}]"),
    Rule(_table_rows_ok, 'Tables require dense hidden axes and nonoverlapping rows'),
    dense_rule('rows', lambda c: (c.dims['m'],), torch.int32, 4),
    dense_rule('q', lambda c: (c.dims['m'], c.dims['k']), torch.int8, 8),
    dense_rule('q_scale', lambda c: (c.dims['m'], 1), torch.float32, 4),
    *_debug_rules(),
    Rule(lambda c: normal_fp32(c.dims['eps']), 'Epsilon must be finite, positive, normal FP32'),
    disjoint_rule(INPUTS, OUTPUTS),
    *_value_rules('shift', ('x', 'weight', 'shift', 'scale')),
]


def validate(x, weight, shift, scale, rows, q, q_scale, *, eps,
             debug_norm=None, debug_rotated=None, debug_rstd=None,
             check_values=True, require_cuda=True):
    """Metadata checks (and, with check_values, the row-map and finiteness scans);
    runnable on CPU tensors with require_cuda=False.  Returns the named (inputs,
    outputs) that a launch owns."""
    names = dict(zip(INPUTS + OUTPUTS, (x, weight, shift, scale, rows, q, q_scale, debug_norm, debug_rotated,
                                        debug_rstd)))
    call = Call(names, {'eps': eps, 'check_values': check_values, 'require_cuda': require_cuda})
    enforce(RULES, call)
    return (tuple((n, names[n]) for n in INPUTS),
            tuple((n, names[n]) for n in OUTPUTS if names[n] is not None))


def require_device(device, what):
    """Raise unless `device` is a B200 and the call runs eagerly (not under torch.compile)."""
    with torch.cuda.device(device):
        if torch.cuda.get_device_capability(device) != DEVICE_CAPABILITY:
            raise RuntimeError('Only the intended B200 (sm_100) device is supported')
        if torch.compiler.is_compiling():
            raise RuntimeError(f'{what} requires eager execution')


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
        report = Resources()
        self.check(self.lib.h3_norm_quant_query_k(k, table_dtype, debug, ct.byref(report), ct.sizeof(report)))
        return {name: int(getattr(report, name)) for name, _ in report._fields_}

    def bind(self, x, weight, shift, scale, rows, q, q_scale, *, eps,
             debug_norm=None, debug_rotated=None, debug_rstd=None, check_values=True):
        inputs, outputs = validate(x, weight, shift, scale, rows, q, q_scale, eps=eps, debug_norm=debug_norm,
                                   debug_rotated=debug_rotated, debug_rstd=debug_rstd, check_values=check_values)
        require_device(x.device, 'NormQuant')
        m, k = x.shape
        ptr = lambda t: None if t is None else t.data_ptr()
        args = [ptr(t) for t in (x, weight, shift, scale, rows, q, q_scale, debug_norm, debug_rotated, debug_rstd)]
        args += [m, k, shift.shape[0], x.stride(0), shift.stride(0), scale.stride(0), float(eps),
                 int(shift.dtype == torch.bfloat16), int(debug_norm is not None)]
        return Bound(self.lib.h3_norm_quant_run_t, x.device, args, [t for _, t in inputs + outputs],
                     [t for _, t in outputs], (q, q_scale), self.check)


Bound = Launch
