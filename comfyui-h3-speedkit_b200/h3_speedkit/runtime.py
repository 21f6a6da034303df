"""Model-scoped B200 backend of the quantized DiT-block linear path.

Mirror of h3_speedkit/runtime.py of H3 SpeedKit for this path: the same class
and function names (``Unsupported``, ``Backend``, ``ModelPatch``,
``patch_model``), the same install flow (clone, explicit block replacements, a
request wrapper, first-use exact verification, fallback to the original block
on ``Unsupported``) and the same error behaviour (checks raise before any
mutation; a launch failure aborts the request, never retried).  Differences:

* the kernels are the sm_100a library (capability 10.0 instead of 12.0), one
  ``libh3sk_b200.so`` published under the reference's library names and checked
  against ``_native/build.json`` (same manifest schema);
* the hidden width K is generic (the reference fixes 5376);
* attention: ``Backend.block(..., attention="int8")`` runs the reference's own
  attention half (runtime.py:129-146): the QKV op's pre-quantised operands, the
  INT8 attention (BSHD, rows below the window zero), the register ConvRot
  quantiser of its output, outproj.  ``attention=None`` is the identity on V of
  the benchmark configuration, and a callable on the BF16 Q/K/V slices of a
  plain QKV projection stays possible.  ``patch_model`` uses "int8" unless told
  otherwise.

ComfyUI and comfy-kitchen are imported lazily, only on the model-patching path.
"""
from __future__ import annotations

import hashlib
import json
import logging
import threading
from collections import Counter
from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass, field
from pathlib import Path

import torch

from . import _lib
from .ops.convrot import ConvRotRegister, quantize_int8_rowwise_convrot64
from .ops.dense import DenseLibrary, allocate_output
from .ops.gemm import int8_gate_residual, int8_linear
from .ops.norm_quant import DEVICE_CAPABILITY, NormQuant

LOG = logging.getLogger(__name__)
KEY = "h3_speedkit_b200"
LIBRARY_NAMES = ("norm", "convrot", "fc1", "gate")
BLOCKS = 50


class Unsupported(ValueError):
    """A contract failed before any in-place model output was changed."""


def verify_manifest(directory: Path) -> dict:
    """Every library name must match its build.json SHA-256 (runtime.py:49-53)."""
    build = json.loads((directory / "build.json").read_text())
    for name in LIBRARY_NAMES:
        path = directory / (name + ".so")
        if not path.exists():
            raise Unsupported("Missing kernel library: " + name)
        if hashlib.sha256(path.read_bytes()).hexdigest() != build["kernels"][name]["sha256"]:
            raise Unsupported("Kernel differs from its build manifest: " + name)
    return build


def segment_rows(segments, tokens: int, table_rows: int, device) -> torch.Tensor:
    """Int32 per-token modulation row map from contiguous (start, stop, row)
    segments (runtime.py:278-291); validated before any GPU work."""
    cursor = 0
    for start, stop, row in segments:
        if (type(start) is not int or type(stop) is not int or type(row) is not int or start != cursor
                or stop < start or not 0 <= row < table_rows):
            raise Unsupported("Only contiguous integer modulation segments are qualified")
        cursor = stop
    if cursor != tokens:
        raise Unsupported("Incomplete modulation row map")
    rows = torch.empty((tokens,), dtype=torch.int32, device=device)
    for start, stop, row in segments:
        rows[start:stop].fill_(row)
    return rows


class Backend:
    """The B200 kernels of one patched model: the manifest-checked library and the
    per-block chain of the linear path (the role of runtime.py:40-164)."""

    def __init__(self, directory=None, *, require_device=True):
        self.directory = Path(directory) if directory else _lib.NATIVE
        if require_device and (not torch.cuda.is_available()
                               or torch.cuda.get_device_capability() != DEVICE_CAPABILITY):
            raise Unsupported("This build requires a B200 (sm_100) GPU")
        self.build = verify_manifest(self.directory)
        library = self.directory / _lib.LIB_NAME
        self.lib = _lib.load(library)
        self.norm = NormQuant(library)
        self.convrot = ConvRotRegister(library)
        from .ops.qkv import QKV
        self.qkv = QKV(self.directory)
        self.dense = DenseLibrary(library)
        # the reference's GEMM entry points by their own names (runtime.py:62-66)
        self.fc1, self.gate = self.lib.h3_int8, self.lib.h3_int8_gate

    @staticmethod
    def plain_weight(module, x):
        """INT8 weight [N, K] and FP32 per-channel scale [N] of a linear module on x's
        device: comfy-kitchen QuantizedTensor weights (runtime.py:97-107) or a module
        that carries ``weight_int8`` / ``weight_scale`` tensors."""
        if hasattr(module, "weight_int8"):
            w, scale = module.weight_int8, module.weight_scale
        else:
            from comfy_kitchen.tensor.int8 import TensorWiseINT8Layout
            w, scale = TensorWiseINT8Layout.get_plain_tensors(module.weight)
        w = w.to(device=x.device).contiguous()
        scale = scale.to(device=x.device, dtype=torch.float32).contiguous().view(-1)
        if w.dtype != torch.int8 or scale.numel() != w.shape[0]:
            raise RuntimeError("Unexpected cast weight layout")
        return w, scale

    def normalize(self, module, x, shift, scale, rows):
        """The fused prologue of `module` (RMSNorm weight, eps) on x: INT8 codes + scales."""
        m, k = x.shape
        q = torch.empty((m, k), device=x.device, dtype=torch.int8)
        qs = torch.empty((m, 1), device=x.device, dtype=torch.float32)
        launch = self.norm.bind(x, module.weight.to(device=x.device).detach(), shift, scale, rows, q, qs,
                                eps=module.eps, check_values=False)
        return launch()

    def gate_projection(self, linear, q, qs, x, gate, rows, skip=0):
        """x[skip:] <- bf(fmaf(bf(dequant(q . W^T)), gate[rows], x)) in place: the
        outproj / FC2 gate-residual GEMM over the rows past the window."""
        if skip >= len(x):
            return
        w, ws = self.plain_weight(linear, x)
        window = slice(skip, None)
        int8_gate_residual(q[window], w, qs[window].reshape(-1), ws, x[window],
                           gate.to(dtype=torch.bfloat16).contiguous(), rows[window])

    def int8_attention(self, block, qi, qs, w, ws, rope, skip):
        """The reference's attention half up to outproj (runtime.py:129-146): the QKV
        op's pre-quantised operands (per-head RMS, RoPE, K anchors, rotation, INT8),
        the INT8 attention from query block skip // 128 on (rows below it zero),
        its BSHD output as [M, heads * 128] BF16."""
        m, dev = qi.shape[0], qi.device
        if rope is None:
            raise Unsupported("INT8 attention needs the block's RoPE table")
        heads = w.shape[0] // (3 * 128)
        qw = block.attn.q_norm.weight.to(device=dev, dtype=torch.bfloat16).contiguous()
        kw = block.attn.k_norm.weight.to(device=dev, dtype=torch.bfloat16).contiguous()
        rope = rope.to(device=dev, dtype=torch.bfloat16).contiguous()
        packed = self.qkv.pack(self.qkv.run(qi, w, qs, ws, rope, qw, kw, float(block.attn.q_norm.eps),
                                            heads=heads), m, heads)
        output = allocate_output(packed, "bshd")
        self.dense.bind(packed, output, start=skip // 128)()
        return output.transpose(1, 2).reshape(m, heads * 128)

    def block(self, block, x, t_emb, segments, rope=None, *, rows, skip=0, counts=None, attention=None,
              mlp_act="gelu_tanh"):
        """One block of the linear path on BF16 tokens x [M, D], updated in place
        (runtime.py:126-164).  attention: "int8" runs the reference's attention
        half (QKV op, INT8 attention, register ConvRot of its output); a callable
        attention(q, k, v) -> [M, D_attn] BF16 takes the slices of a plain QKV
        projection; None is the identity on V (the benchmark configuration).
        mlp_act: 'gelu_tanh' (FC1 epilogue, the benchmark configuration) or
        'swiglu' (the H3 geometry: FC1 rows are [gate | up])."""
        counts = Counter() if counts is None else counts
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = block.adaln_proj(t_emb)
        qi, qs = self.normalize(block.norm1, x, shift_msa, scale_msa, rows)
        w, ws = self.plain_weight(block.attn.qkv_proj, x)
        if attention == "int8":
            attn = self.int8_attention(block, qi, qs, w, ws, rope, skip)
            aq = torch.empty(attn.shape, device=x.device, dtype=torch.int8)
            asc = torch.empty((len(x), 1), device=x.device, dtype=torch.float32)
            self.convrot.bind(attn, aq, asc, check_finite=False)()
        else:
            qkv = int8_linear(qi, w, qs, ws)
            width = qkv.shape[1] // 3
            q_, k_, v_ = qkv[:, :width], qkv[:, width:2 * width], qkv[:, 2 * width:]
            attn = v_ if attention is None else attention(q_, k_, v_)
            aq, asc = quantize_int8_rowwise_convrot64(attn)
        self.gate_projection(block.attn.out_proj, aq, asc, x, gate_msa, rows, skip)
        qi, qs = self.normalize(block.norm2, x, shift_mlp, scale_mlp, rows)
        w1, ws1 = self.plain_weight(block.mlp.fc1, x)
        # FC1 only for the rows past the window; the rows below it stay zero
        # (runtime.py:149-157)
        hidden = torch.empty((len(x), w1.shape[0]), device=x.device, dtype=torch.bfloat16)
        if skip:
            hidden[:skip].zero_()
        if skip < len(x):
            int8_linear(qi[skip:], w1, qs[skip:], ws1, gelu=mlp_act != "swiglu", out=hidden[skip:])
        if mlp_act == "swiglu":
            fq, fs = quantize_int8_rowwise_convrot64(hidden, 256, input_act="swiglu")
        else:
            fq, fs = quantize_int8_rowwise_convrot64(hidden)
        self.gate_projection(block.mlp.fc2, fq, fs, x, gate_mlp, rows, skip)
        counts.update(qkv=1, attention=1, norm_quant=2, fc1=1, gate=2)
        if skip:
            counts.update(last_block_window=1)
        return x


def last_block_window(payload, tokens: int) -> int:
    """The last block's row window (runtime.py:205-215): the first target
    (video/audio) token rounded down to 128, when the prepared layout holds two
    contiguous target spans that end the sequence; 0 (every row) otherwise."""
    layout = payload.get("layout") if isinstance(payload, dict) else None
    if layout is None or getattr(layout, "seq_len", None) != tokens:
        return 0
    targets = [(a, b) for a, b, kind in layout.segments if kind in ("video", "audio")]
    if len(targets) != 2 or targets[-1][1] != tokens or targets[0][1] != targets[1][0]:
        return 0
    return min(a for a, _ in targets) // 128 * 128


@dataclass
class RequestFrame:
    """State of one sampler call through the patched model (one diffusion-model
    evaluation): set by the request wrapper, read by every block replacement."""
    tokens: int = 0
    skip: int = 0
    shape_key: tuple = ()
    verify: bool = False
    counts: Counter = field(default_factory=Counter)
    rows: torch.Tensor | None = None
    row_key: tuple | None = None
    fallback: str | None = None
    verification_failed: int | None = None

    @property
    def active(self) -> bool:
        return self.fallback is None and self.verification_failed is None

    def rows_for(self, segments, tokens, table_rows, device):
        """The int32 row map of `segments`, rebuilt only when the segments change."""
        key = tuple(segments)
        if self.row_key != key:
            self.rows, self.row_key = segment_rows(segments, tokens, table_rows, device), key
        return self.rows

    def report(self) -> dict:
        """The last_report record: every field that is set, counters as plain dicts."""
        out = {}
        for name in ("tokens", "skip", "shape_key", "verify", "counts", "fallback", "verification_failed"):
            value = getattr(self, name)
            if value is not None:
                out[name] = dict(value) if isinstance(value, Counter) else value
        return out


class BlockReplacement:
    """The ``("double_block", index)`` replacement ComfyUI calls as run(inputs, extra)."""

    def __init__(self, patch, index):
        self.patch, self.index = patch, index

    def __call__(self, inputs, extra):
        frame = self.patch.context.get()
        if frame is None or not frame.active:
            return extra["original_block"](inputs)
        return self.patch.run_block(frame, self.index, inputs, extra)


class ModelPatch:
    """Request wrapper + block replacements (the roles of runtime.py:167-308)."""

    def __init__(self, model, backend, verify_new_shapes=True, attention="int8", blocks=BLOCKS):
        self.model = model
        self.backend = backend
        self.attention = attention
        self.blocks = blocks
        self.context = ContextVar("speedkit_b200_request", default=None)
        self.lock = threading.RLock()
        self.last_report = {}
        self.warned = set()
        self.verify_new_shapes = verify_new_shapes
        self.verified_shapes = Counter()
        self.rejected_shapes = set()

    def preflight(self, args, kwargs) -> RequestFrame:
        """Checks that run before any block; raises Unsupported (nothing mutated yet)."""
        if torch.is_grad_enabled():
            raise Unsupported("Eager inference only")
        first = args[0] if args else None
        x = first[0] if isinstance(first, (list, tuple)) else first
        if x is None or not x.is_cuda or torch.cuda.get_device_capability(x.device) != DEVICE_CAPABILITY:
            raise Unsupported("B200 GPU required")
        if self.attention is None:
            raise Unsupported("No attention provider for the B200 linear path")
        tokens = int(x.shape[-2]) if x.ndim >= 2 else 0
        payload = kwargs.get("minimax_payload") or (args[4] if len(args) > 4 else None)
        skip = last_block_window(payload, tokens)
        key = (tokens, skip)
        return RequestFrame(tokens=tokens, skip=skip, shape_key=key,
                            verify=self.verify_new_shapes and self.verified_shapes[key] < 8)

    def _open(self, args, kwargs) -> RequestFrame:
        try:
            return self.preflight(args, kwargs)
        except Unsupported as error:
            reason = str(error)
            if reason not in self.warned:       # one warning per distinct reason
                self.warned.add(reason)
                LOG.warning("H3 SpeedKit fallback: %s", reason)
            return RequestFrame(fallback=reason)

    @contextmanager
    def _request(self, args, kwargs):
        frame = self._open(args, kwargs)
        token = self.context.set(frame)
        try:
            yield frame
        finally:
            self.context.reset(token)

    def _close(self, frame: RequestFrame) -> None:
        if frame.fallback is None and frame.counts["attention"] != self.blocks:
            raise RuntimeError("Incomplete SpeedKit block coverage")
        if frame.verify and frame.verification_failed is None:
            self.verified_shapes[frame.shape_key] += 1
        self.last_report = frame.report()

    def wrapper(self, executor, *args, **kwargs):
        """The DIFFUSION_MODEL wrapper: one request frame around the executor."""
        with self.lock, self._request(args, kwargs) as frame:
            result = executor(*args, **kwargs)
            self._close(frame)
            return result

    def replacement(self, index):
        return BlockReplacement(self, index)

    def run_block(self, frame: RequestFrame, index: int, inputs, extra):
        """Block `index` on the B200 path.  In a verifying request the block runs on a
        private clone beside the original block, and a single differing bit (rows
        the last block's window skips excepted) rejects the layout and returns the
        original block's result."""
        x = inputs["img"]
        if x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise RuntimeError("Hidden activation changed after preflight")
        rows = frame.rows_for(inputs["mod_segments"], len(x), inputs["t_emb"].shape[0] * 3, x.device)
        window = frame.skip if index == self.blocks - 1 else 0   # the final layer reads rows [skip, M)
        work = x.clone() if frame.verify else x
        expected = extra["original_block"](inputs)["img"] if frame.verify else None
        out = self.backend.block(self.model.blocks[index], work, inputs["t_emb"], inputs["mod_segments"],
                                 inputs.get("rope_freqs"), rows=rows, skip=window, counts=frame.counts,
                                 attention=self.attention)
        if expected is None or torch.equal(out[window:], expected[window:]):
            return {"img": out}
        self.rejected_shapes.add(frame.shape_key)
        frame.verification_failed = index
        frame.fallback = "Exact layout verification failed at block " + str(index)
        LOG.warning("H3 SpeedKit: %s; using reference", frame.fallback)
        return {"img": expected}


def patch_model(model, directory=None, *, release_embeddings=True, verify_new_shapes=True, attention="int8",
                backend=None):
    """Return a Comfy clone with explicit block replacements and a request
    wrapper (runtime.py:311-338).  The original model is not modified.
    attention: "int8" (the reference's QKV op and INT8 attention, the default) or
    a callable provider on the BF16 Q/K/V slices; None (identity) is refused."""
    import comfy.patcher_extension as pe
    if attention is None:
        raise Unsupported("The B200 path needs an attention provider: 'int8' or a callable (None is identity)")
    clone = model.clone()
    options = clone.model_options.setdefault("transformer_options", {})
    existing = options.get("patches_replace", {}).get("dit", {})
    if any(("double_block", i) in existing for i in range(BLOCKS)):
        raise Unsupported("A DiT block replacement is already installed; start from the unpatched MODEL output")
    patch = ModelPatch(model.model.diffusion_model, backend or Backend(directory), verify_new_shapes, attention)
    for index in range(BLOCKS):
        clone.set_model_patch_replace(patch.replacement(index), "dit", "double_block", index)
    pe.add_wrapper_with_key(pe.WrappersMP.DIFFUSION_MODEL, KEY, patch.wrapper,
                            clone.model_options["transformer_options"])
    clone._h3_speedkit = patch
    return clone
