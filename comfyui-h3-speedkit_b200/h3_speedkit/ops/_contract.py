"""Operand contracts of the row-kernel bindings, stated as data.

Each binding (``norm_quant``, ``residual_quant``, ``convrot``) describes its C
entry point's operand contract as an ordered list of ``Rule`` objects: a
predicate over a ``Call`` (the named operands plus the dimensions taken from the
leading operand) and the error text a caller sees when it fails.  ``enforce``
walks the list and raises ``ValueError`` at the first broken rule, so the order
of the list is the order in which a caller learns about problems.  The error
texts are the interface the reference's bindings expose
(h3_speedkit/ops/norm_quant.py:57-105, ops/residual_quant.py:57-112,
ops/convrot.py:60-92 of H3 SpeedKit) and are kept word for word; everything
else here is this package's own structure.

``Launch`` is the one validated-call object all three bindings return from
``bind``: it owns every operand tensor, records their use on the current stream
before the launch, marks the written tensors as modified, and turns a nonzero
``cudaError_t`` into ``RuntimeError`` (the request is aborted, never retried:
stores may already be queued when the error is reported).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch

INT32_MAX = 0x7fffffff
FP32_TINY = torch.finfo(torch.float32).tiny
FP32_MAX = torch.finfo(torch.float32).max


@dataclass
class Call:
    """Named operands of one call and the dimensions read off its leading operand."""
    operands: dict
    dims: dict = field(default_factory=dict)

    def __getitem__(self, name):
        return self.operands[name]

    def present(self):
        return [(n, t) for n, t in self.operands.items() if t is not None]


@dataclass(frozen=True)
class Rule:
    ok: Callable[[Call], bool]
    message: str | Callable[[Call], str]

    def text(self, call: Call) -> str:
        return self.message(call) if callable(self.message) else self.message


def enforce(rules: Sequence[Rule], call: Call) -> None:
    for rule in rules:
        if not rule.ok(call):
            raise ValueError(rule.text(call))


# ---- predicates ---------------------------------------------------------------------

def address_range(t: torch.Tensor) -> tuple[int, int]:
    """[first byte, one past the last byte] that a strided tensor can reach."""
    if t.numel() == 0:
        return t.data_ptr(), t.data_ptr()
    reach = 1 + sum((n - 1) * s for n, s in zip(t.shape, t.stride()))
    return t.data_ptr(), t.data_ptr() + reach * t.element_size()


def first_overlap(inputs, outputs):
    """An (output, other, other_is_output) pair whose address ranges intersect, or None.

    One sweep over the ranges sorted by their first byte: each range is compared
    only with the ranges still open where it starts, and a pair counts when at
    least one side is an output (inputs may share memory).  Empty tensors reach
    no memory and never overlap."""
    spans = sorted((*address_range(t), name, is_out)
                   for group, is_out in ((outputs, True), (inputs, False)) for name, t in group)
    open_spans = []
    for lo, hi, name, is_out in spans:
        if hi <= lo:
            continue
        open_spans = [s for s in open_spans if s[1] > lo]
        for _, _, other, other_out in open_spans:
            if is_out or other_out:
                if not is_out:   # name the output first
                    return other, name, False
                return name, other, other_out
        open_spans.append((lo, hi, name, is_out))
    return None


def all_finite(t: torch.Tensor, chunk_rows: int = 128) -> bool:
    """NaN/Inf scan in bounded row chunks (no full-size temporary)."""
    parts = (t,) if t.ndim < 2 else torch.split(t, chunk_rows, dim=0)
    return all(bool(torch.isfinite(p).all().item()) for p in parts)


def normal_fp32(value) -> bool:
    v = float(value)
    return math.isfinite(v) and FP32_TINY <= v <= FP32_MAX


def is_dense(t, shape, dtype, alignment) -> bool:
    return (tuple(t.shape) == tuple(shape) and t.dtype == dtype and t.is_contiguous()
            and t.data_ptr() % alignment == 0)


def dense_rule(name: str, dims: Callable[[Call], tuple], dtype, alignment: int) -> Rule:
    """Contiguous `dtype` tensor of shape dims(call), `alignment`-byte aligned."""
    return Rule(lambda c: is_dense(c[name], dims(c), dtype, alignment),
                lambda c: f'{name} requires contiguous {dtype} {tuple(dims(c))} and {alignment}B alignment')


def common_rules(require_cuda_of: str) -> list[Rule]:
    """Rules every row-kernel call starts with: plain tensors on one CUDA device,
    nothing that records autograd history."""
    return [
        Rule(lambda c: all(type(t) is torch.Tensor for _, t in c.present()),
             'All operands must be original plain Torch tensors'),
        Rule(lambda c: (not c.dims.get('require_cuda', True) or c[require_cuda_of].is_cuda)
             and len({t.device for _, t in c.present()}) == 1,
             'All operands must use one CUDA device'),
        Rule(lambda c: not any(t.requires_grad for _, t in c.present()),
             'Inference only; detach only after validating model autograd policy'),
    ]


def debug_rule(names=('debug_norm', 'debug_rotated', 'debug_rstd')) -> Rule:
    return Rule(lambda c: len({c[n] is None for n in names}) == 1,
                'Debug requires norm, rotated, and rstd outputs together')


def disjoint_rule(inputs: Sequence[str], outputs: Sequence[str]) -> Rule:
    def verdict(c):
        ins = [(n, c[n]) for n in inputs if c[n] is not None]
        outs = [(n, c[n]) for n in outputs if c[n] is not None]
        return first_overlap(ins, outs)

    def message(c):
        out, other, other_is_output = verdict(c)
        return f'Outputs {out} and {other} overlap' if other_is_output else f'Output {out} overlaps input {other}'
    return Rule(lambda c: verdict(c) is None, message)


# ---- the validated call -------------------------------------------------------------

class Launch:
    """One validated call of a C entry point (the ``Bound`` object of the reference's
    bindings): ``launch()`` / ``launch.__call__()`` enqueues it on the device's current
    stream and returns ``result``.

    entry     the ctypes function; called as entry(*args, stream_handle)
    owners    every tensor the call reads or writes (kept alive, stream-recorded)
    written   the tensors the call writes (their autograd versions are bumped)
    check     maps the C return code to success or a raised RuntimeError
    """

    def __init__(self, entry, device, args, owners, written, result, check):
        self.entry, self.device, self.args = entry, device, list(args)
        self.owners = tuple(t for t in owners if t is not None)
        self.written = tuple(t for t in written if t is not None)
        self.result, self._check = result, check

    def __call__(self):
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device)
            for t in self.owners:
                t.record_stream(stream)
            code = self.entry(*self.args, stream.cuda_stream)
            if self.written:
                torch.autograd.graph.increment_version(self.written)
            self._check(code)
        return self.result
