"""Current-stream binding of the INT8 attention (B200) on the QKV op's operands.

Stands in for h3_speedkit/ops/dense.py of H3 SpeedKit: the same names
(``DenseArgs``, ``DenseLibrary``, ``allocate_output``, ``BoundDense``), argument
meaning and error texts, over ``h3_dense_*`` of libh3sk_b200.so (the tcgen05
kernel with the reference's arithmetic).  ``DenseLibrary.bind`` takes the
``PrequantizedInt8Attention`` fields (q, k, v codes and their scales, as
``ops.qkv.QKV`` returns them) and an output tensor, checks the layouts the C
entry point requires, and returns a callable that launches on the current stream.
"""
from __future__ import annotations

import ctypes as ct

import torch

from .. import _lib

_POINTERS = ("q", "k", "v", "o", "q_scale", "k_scale", "v_scale")
_SIZES = ("batch", "qo_len", "kv_len", "qo_heads", "kv_heads", "q_stride_b", "q_stride_h", "q_stride_s",
          "k_stride_b", "k_stride_h", "k_stride_s", "v_stride_b", "v_stride_h", "v_stride_d",
          "o_stride_b", "o_stride_h", "o_stride_s")


class DenseArgs(ct.Structure):
    """The C argument block H3DenseArgs (include/h3sk_b200.h; dense_ring.cu:16-24)."""
    _fields_ = [(n, ct.c_void_p) for n in _POINTERS] + [(n, ct.c_uint32) for n in _SIZES] + \
        [("sm_scale", ct.c_float)]


def allocate_output(packed, layout="bhsd"):
    """BF16 output with the logical shape of q [B, H, S, D]; "bshd" stores it
    token-major (a transposed view), so a [B, S, H*D] reshape is free."""
    b, h, s, d = packed.q.shape
    if layout == "bhsd":
        return torch.empty((b, h, s, d), dtype=torch.bfloat16, device=packed.q.device)
    if layout == "bshd":
        return torch.empty((b, s, h, d), dtype=torch.bfloat16, device=packed.q.device).transpose(1, 2)
    raise ValueError(f"Unsupported output layout: {layout}")


def _layout_errors(packed, output):
    """The reference binding's checks (ops/dense.py:61-91) as (failed, message) pairs, in order."""
    q, k, v = packed.q, packed.k, packed.v
    scales = (packed.q_scale, packed.k_scale, packed.v_scale)
    tensors = (q, k, v, *scales, output)
    yield (any(not t.is_cuda or t.device != q.device for t in tensors),
           "Packed input/output devices must agree")
    yield (packed.cta_k != 128 or q.shape[-1] != 128 or packed.original_head_dim != 128,
           "This build only supports the observed D128/CTA_K128 path")
    yield (packed.input_dtype != torch.bfloat16 or output.dtype != torch.bfloat16,
           "This strict replay only supports the captured BF16 path")
    yield (packed.attn_mask is not None or output.shape != q.shape,
           "Only unmasked BHSD logical outputs are supported")
    yield (any(t.dtype != torch.int8 for t in (q, k, v)), "Q/K/V must retain the original INT8 carrier")
    yield (any(t.dtype != torch.float32 for t in scales), "Quantization scales must be FP32")
    yield (any(not t.is_contiguous() for t in tensors[:-1]) or output.stride(-1) != 1,
           "Packed inputs must use the exact contiguous Kitchen ABI")


class DenseLibrary:
    """ctypes front of h3_dense_* (libh3sk_b200.so, published as dense.so)."""

    def __init__(self, path=None):
        self.lib = _lib.load(path)
        if self.lib.h3_dense_args_size() != ct.sizeof(DenseArgs):
            raise RuntimeError("C/ctypes ABI struct size mismatch")
        self.group = self.lib.h3_dense_query_group()

    def bind(self, packed, output, *, start=0):
        for failed, message in _layout_errors(packed, output):
            if failed:
                raise ValueError(message)
        q, k, v = packed.q, packed.k, packed.v
        b, h, s, d = q.shape
        hk, sk = k.shape[1:3]
        padded = (sk + 127) // 128 * 128
        if k.shape[0] != b or k.shape[-1] != d or h % hk:
            raise ValueError("Invalid Q/K heads or dimensions")
        if tuple(v.shape) != (b * hk * d, padded):
            raise ValueError("V must use Kitchen's [B*Hkv*D, padded_Sk] layout")
        if tuple(packed.q_scale.shape) != (b, h, (s + 127) // 128 * 32):
            raise ValueError("Invalid D128 per-thread Q scale layout")
        if tuple(packed.k_scale.shape) != (b, hk, (sk + 127) // 128 * 4):
            raise ValueError("Invalid per-thread K scale layout")
        if packed.v_scale.numel() != b * hk * d:
            raise ValueError("Invalid V scale layout")
        if tuple(output.stride()) not in ((h * s * d, s * d, d, 1), (s * h * d, d, h * d, 1)):
            raise ValueError("Output must be BHSD or BSHD storage without overlap")
        sizes = (b, s, sk, h, hk, *q.stride()[:3], *k.stride()[:3], hk * d * padded, d * padded, padded,
                 *output.stride()[:3])
        if any(x < 0 or x > 0x7fffffff for x in sizes):
            raise ValueError("Shape/stride exceeds the upstream int32 ABI")
        ptrs = (q, k, v, output, packed.q_scale, packed.k_scale, packed.v_scale)
        args = DenseArgs(*(t.data_ptr() for t in ptrs), *sizes, float(packed.attention_scale))
        return BoundDense(self, ptrs, args, output, start)


class BoundDense:
    """A checked launch: owns its tensors and argument block."""

    def __init__(self, library, owners, args, output, start):
        self.library, self.owners, self.params, self.output, self.start = library, owners, args, output, start

    def __call__(self):
        with torch.cuda.device(self.output.device):
            stream = torch.cuda.current_stream(self.output.device)
            for t in self.owners:
                t.record_stream(stream)
            code = self.library.lib.h3_dense_launch_window(ct.byref(self.params), stream.cuda_stream, self.start)
        if code:
            raise RuntimeError(f"Dense CUDA launch failed ({code}): "
                               + self.library.lib.h3_dense_error_string(code).decode())
        return self.output
