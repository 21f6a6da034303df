"""Host-side contracts on CPU: binding validation, row maps, manifest checks,
model patching and the request wrapper (with fake ComfyUI modules, in the style
of the reference's tests/test_indexed_gate.py)."""
import copy
import json
import shutil
import sys
from types import ModuleType, SimpleNamespace
from unittest.mock import patch

import pytest
import torch

from h3_speedkit import runtime
from h3_speedkit.ops import norm_quant as nq
from h3_speedkit.runtime import Unsupported


def _operands(m=4, k=512, tables=2, dtype=torch.bfloat16):
    x = torch.randn((m, k)).to(torch.bfloat16)
    w = torch.ones((k,), dtype=torch.bfloat16)
    shift = torch.zeros((tables, k), dtype=dtype)
    scale = torch.zeros((tables, k), dtype=dtype)
    rows = torch.zeros((m,), dtype=torch.int32)
    q = torch.empty((m, k), dtype=torch.int8)
    qs = torch.empty((m, 1), dtype=torch.float32)
    return x, w, shift, scale, rows, q, qs


def test_validate_accepts_the_contract_on_cpu():
    ins, outs = nq.validate(*_operands(), eps=1e-6, require_cuda=False)
    assert [n for n, _ in ins] == ["x", "weight", "shift", "scale", "rows"]
    ins, outs = nq.validate(*_operands(dtype=torch.float32), eps=1e-6, require_cuda=False)


@pytest.mark.parametrize("mutate, message", [
    (lambda o: o.__setitem__(0, o[0].float()), "X requires"),
    (lambda o: o.__setitem__(0, torch.randn((4, 500)).to(torch.bfloat16)), "X requires"),
    (lambda o: o.__setitem__(1, torch.ones((256,), dtype=torch.bfloat16)), "weight requires"),
    (lambda o: o.__setitem__(3, torch.zeros((2, 512), dtype=torch.float32)), "Tables require"),
    (lambda o: o.__setitem__(4, torch.zeros((4,), dtype=torch.int64)), "rows requires"),
    (lambda o: o.__setitem__(5, torch.empty((4, 512), dtype=torch.uint8)), "q requires"),
    (lambda o: o.__setitem__(6, torch.empty((4,), dtype=torch.float32)), "q_scale requires"),
])
def test_validate_rejects(mutate, message):
    ops = list(_operands())
    mutate(ops)
    with pytest.raises(ValueError, match=message):
        nq.validate(*ops, eps=1e-6, require_cuda=False)


def test_validate_rejects_bad_eps_overlap_nonfinite_and_rows():
    x, w, shift, scale, rows, q, qs = _operands()
    for eps in (0.0, float("nan"), float("inf"), 1e-45):
        with pytest.raises(ValueError, match="Epsilon"):
            nq.validate(x, w, shift, scale, rows, q, qs, eps=eps, require_cuda=False)
    alias = x.view(torch.int8)[:, :512]
    with pytest.raises(ValueError):
        nq.validate(x, w, shift, scale, rows, alias, qs, eps=1e-6, require_cuda=False)
    bad = x.clone()
    bad[2, 7] = float("nan")
    with pytest.raises(ValueError, match="Nonfinite"):
        nq.validate(bad, w, shift, scale, rows, q, qs, eps=1e-6, require_cuda=False)
    rows_bad = torch.full((4,), 2, dtype=torch.int32)
    with pytest.raises(ValueError, match="Rows outside"):
        nq.validate(x, w, shift, scale, rows_bad, q, qs, eps=1e-6, require_cuda=False)


def test_debug_outputs_come_together():
    x, w, shift, scale, rows, q, qs = _operands()
    with pytest.raises(ValueError, match="Debug requires"):
        nq.validate(x, w, shift, scale, rows, q, qs, eps=1e-6, require_cuda=False,
                    debug_norm=torch.empty((4, 512), dtype=torch.bfloat16))


def test_check_disjoint_and_span_include_strided_padding():
    base = torch.zeros((4, 16))
    a = base[:, :8]
    assert nq.span(a) == (a.data_ptr(), a.data_ptr() + (3 * 16 + 8) * 4)
    with pytest.raises(ValueError, match="overlap"):
        nq.check_disjoint([("a", a)], [("b", base[3:, 4:])])
    nq.check_disjoint([("a", base[:2])], [("b", base[2:])])


def test_segment_rows_reject_before_gpu_work():
    assert runtime.segment_rows([(0, 3, 0), (3, 3, 1), (3, 8, 2)], 8, 3, "cpu").tolist() == [0, 0, 0, 2, 2, 2, 2, 2]
    for segments in ([(0, 4, 0), (5, 8, 1)], [(0, 5, 0), (4, 8, 1)], [(0, 8, -1)], [(0, 8, 3)], [(0, 9, 0)],
                     [(0, 7, 0)], [(0, 8, [0])], [(0, 8, True)]):
        with pytest.raises(Unsupported):
            runtime.segment_rows(segments, 8, 3, "cpu")


def test_manifest_sha_mismatch_is_unsupported(tmp_path):
    from h3_speedkit import _lib
    for name in ("build.json", _lib.LIB_NAME):
        shutil.copy(_lib.NATIVE / name, tmp_path / name)
    for alias in runtime.LIBRARY_NAMES:
        (tmp_path / (alias + ".so")).symlink_to(_lib.LIB_NAME)
    runtime.verify_manifest(tmp_path)
    build = json.loads((tmp_path / "build.json").read_text())
    build["kernels"]["gate"]["sha256"] = "0" * 64
    (tmp_path / "build.json").write_text(json.dumps(build))
    with pytest.raises(Unsupported, match="gate"):
        runtime.verify_manifest(tmp_path)
    (tmp_path / "fc1.so").unlink()
    with pytest.raises(Unsupported, match="fc1"):
        runtime.verify_manifest(tmp_path)


def test_backend_requires_a_b200():
    if torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0):
        pytest.skip("a B200 is present")
    with pytest.raises(Unsupported, match="B200"):
        runtime.Backend()


def _copy_options(obj):
    if isinstance(obj, dict):
        return {key: _copy_options(value) for key, value in obj.items()}
    if isinstance(obj, list):
        return [_copy_options(value) for value in obj]
    return obj


class FakeModel:
    def __init__(self):
        self.model_options = {"transformer_options": {"keep": "original"}}
        self.model = SimpleNamespace(diffusion_model=SimpleNamespace(blocks=[]))

    def clone(self):
        cloned = copy.copy(self)
        cloned.model_options = _copy_options(self.model_options)
        return cloned

    def set_model_patch_replace(self, replacement, name, block, index):
        # ComfyUI replaces this options dictionary on every call
        options = _copy_options(self.model_options["transformer_options"])
        options.setdefault("patches_replace", {}).setdefault(name, {})[(block, index)] = replacement
        self.model_options["transformer_options"] = options


def _fake_comfy():
    modules = {name: ModuleType(name) for name in ("comfy", "comfy.patcher_extension")}
    modules["comfy"].patcher_extension = modules["comfy.patcher_extension"]
    pe = modules["comfy.patcher_extension"]
    pe.WrappersMP = SimpleNamespace(DIFFUSION_MODEL="diffusion")
    pe.add_wrapper_with_key = lambda kind, key, wrapper, options: options.setdefault("wrappers", {}).update(
        {key: wrapper})
    return modules


def test_patch_model_installs_on_a_clone_and_rejects_double_install():
    model = FakeModel()
    with patch.dict(sys.modules, _fake_comfy()):
        with pytest.raises(Unsupported, match="attention provider"):
            runtime.patch_model(model, attention=None)
        assert runtime.patch_model(model, backend=object())._h3_speedkit.attention == "int8"
        fast = runtime.patch_model(model, attention=lambda q, k, v: v, backend=object())
        assert model.model_options == {"transformer_options": {"keep": "original"}}
        options = fast.model_options["transformer_options"]
        assert len(options["patches_replace"]["dit"]) == runtime.BLOCKS
        assert options["wrappers"][runtime.KEY].__self__ is fast._h3_speedkit
        with pytest.raises(Unsupported, match="already installed"):
            runtime.patch_model(fast, attention=lambda q, k, v: v, backend=object())


def test_wrapper_falls_back_and_cleans_context():
    consumer = runtime.ModelPatch(object(), backend=object())

    def executor(*args, **kwargs):
        assert consumer.context.get().fallback is not None
        return "original result"
    with patch.object(runtime.LOG, "warning") as warn:
        assert consumer.wrapper(executor, [torch.zeros((1, 4))]) == "original result"
        assert warn.called
    assert consumer.context.get() is None
    assert "fallback" in consumer.last_report

    def failed(*args, **kwargs):
        raise OSError("executor failure")
    with pytest.raises(OSError):
        consumer.wrapper(failed, [torch.zeros((1, 4))])
    assert consumer.context.get() is None

    # a replacement outside a request, or in a fallback request, runs the original block
    run = consumer.replacement(0)
    assert run({"img": 1}, {"original_block": lambda inputs: "orig"}) == "orig"


def test_node_schema_matches_the_reference():
    io = ModuleType("comfy_api.latest.io")

    class Spec(SimpleNamespace):
        pass

    class Kind:
        def __init__(self, name):
            self.name = name

        def Input(self, *a, **k):
            return Spec(kind=self.name, args=a, kw=k)

        def Output(self, *a, **k):
            return Spec(kind=self.name, args=a, kw=k)

    io.ComfyNode = object
    io.Schema = lambda **kw: Spec(**kw)
    io.Model, io.Boolean, io.String = Kind("model"), Kind("bool"), Kind("string")
    io.NodeOutput = lambda *a: a
    latest = ModuleType("comfy_api.latest")
    latest.io = io
    modules = {"comfy_api": ModuleType("comfy_api"), "comfy_api.latest": latest}
    with patch.dict(sys.modules, modules):
        from h3_speedkit import nodes
        (node,) = nodes.make_nodes()
        schema = node.define_schema()
        assert schema.node_id == "H3SpeedKitOptimize"
        assert [i.kind for i in schema.inputs] == ["model", "bool"]
        assert [o.kind for o in schema.outputs] == ["model", "string"]
        out = node.execute(FakeModel(), enabled=False)
        assert out[1] == "H3 SpeedKit disabled"


def test_block_geometry_from_weight_shapes():
    from h3_speedkit import synthetic
    from h3_speedkit.stack import geometry
    g = geometry(synthetic.cfg5_block(0, 512, 1024))
    assert g == {"d": 512, "attn": 512, "ffn": 1024, "fc1_n": 1024, "swiglu": False}
    g = geometry(synthetic.cfg5_block(0, 512, 512, attn=768, swiglu=True))
    assert g == {"d": 512, "attn": 768, "ffn": 512, "fc1_n": 1024, "swiglu": True}
    b = synthetic.cfg5_block(0, 512, 512, attn=768, swiglu=True)
    b.out = b.out[:, :512]
    with pytest.raises(ValueError):
        geometry(b)


@pytest.mark.parametrize("swiglu", [False, True])
def test_block_plan_launch_lists(swiglu):
    """The block plan's launches, bound on CPU tensors (nothing is launched):
    with epilogue rotation the QKV GEMM rotates its V third (rot_n0 = 2 attn)
    for the V codes pass, and in GELU blocks FC1 rotates all of h for the FC2
    codes pass; SwiGLU blocks keep FC1 + the SwiGLU quantiser.  Without it, the
    GEMMs are followed by the full quantisers."""
    from h3_speedkit import _lib, synthetic
    from h3_speedkit.stack import BlockPlan, Workspace
    d, ffn, attn, m, skip = 512, 512, 768, 384, 128
    b = synthetic.cfg5_block(0, d, ffn, attn=attn, swiglu=swiglu)
    x = torch.zeros((m, d), dtype=torch.bfloat16)
    rows = torch.zeros((m,), dtype=torch.int32)
    ws = Workspace.for_block(m, b, "cpu")
    lib = _lib.load()
    fused = BlockPlan(b, x, rows, ws, skip=skip)
    names = [(name, fn.__name__) for name, fn, _ in fused.calls]
    assert names == [("prologue", "h3_norm_quant_run_t"), ("qkv", "h3_int8_rot"),
                     ("quant_v", "h3_convrot_codes"), ("outproj", "h3_int8_gate"),
                     ("prologue", "h3_norm_quant_run_t"),
                     ("fc1", "h3_int8_ex" if swiglu else "h3_int8_gelu_rot"),
                     ("quant_h", "h3_convrot_quant_act" if swiglu else "h3_convrot_codes"),
                     ("fc2", "h3_int8_gate")]
    qkv_args = fused.calls[1][2]
    assert qkv_args[-2:] == (0, 2 * attn)                 # plain dequant, V third rotated
    assert qkv_args[6] == ws.vmax.data_ptr()              # row maxima of all m rows
    quant_v_args = fused.calls[2][2]
    assert quant_v_args[2] == ws.vmax.data_ptr() + 4 * skip   # the window's rows only
    assert quant_v_args[5:] == (m - skip, attn)
    plain = BlockPlan(b, x, rows, ws, skip=skip, epilogue_rotation=False)
    names = [(name, fn.__name__) for name, fn, _ in plain.calls]
    assert [n for n, _ in names] == [c[0] for c in fused.calls]
    assert dict(names)["qkv"] == "h3_int8_ex"
    assert names[2] == ("quant_v", "h3_convrot_quant_act")
    assert names[6] == ("quant_h", "h3_convrot_quant_act")
    assert lib is _lib.load()


def test_residual_validate_rejects_before_gpu_work():
    """ops.residual_quant.validate: the reference's metadata checks (residual_quant.py:57-112) on CPU."""
    from h3_speedkit.ops import residual_quant as rq
    m, k = 4, 512
    x = torch.zeros((m, k), dtype=torch.bfloat16)
    branch = torch.zeros_like(x)
    w = torch.ones((k,), dtype=torch.bfloat16)
    gate = torch.zeros((2, k))
    shift = torch.zeros((2, k), dtype=torch.bfloat16)
    scale = torch.zeros_like(shift)
    rows = torch.zeros((m,), dtype=torch.int32)
    q = torch.empty((m, k), dtype=torch.int8)
    qs = torch.empty((m, 1))
    ok = dict(eps=1e-6, require_cuda=False)
    rq.validate(x, branch, w, gate, shift, scale, rows, q, qs, **ok)
    with pytest.raises(ValueError, match="overlaps"):
        rq.validate(x, x, w, gate, shift, scale, rows, q, qs, **ok)
    with pytest.raises(ValueError, match="Branch requires"):
        rq.validate(x, branch[:, :256], w, gate, shift, scale, rows, q, qs, **ok)
    with pytest.raises(ValueError, match="Gate requires"):
        rq.validate(x, branch, w, gate[:1], shift, scale, rows, q, qs, **ok)
    with pytest.raises(ValueError, match="Rows outside"):
        rq.validate(x, branch, w, gate, shift, scale, rows + 2, q, qs, **ok)
    with pytest.raises(ValueError, match="Nonfinite"):
        bad = branch.clone()
        bad[1, 3] = float("inf")
        rq.validate(x, bad, w, gate, shift, scale, rows, q, qs, **ok)
    with pytest.raises(ValueError, match="Epsilon"):
        rq.validate(x, branch, w, gate, shift, scale, rows, q, qs, eps=0.0, require_cuda=False)


def test_last_block_window_from_the_prepared_layout():
    """runtime.py:205-215: the first target token rounded down to 128 when two
    contiguous target spans end the sequence; 0 otherwise."""
    lay = SimpleNamespace(seq_len=5000, segments=[(0, 700, "text"), (700, 4000, "video"), (4000, 5000, "audio")])
    assert runtime.last_block_window({"layout": lay}, 5000) == 640
    assert runtime.last_block_window({"layout": lay}, 4999) == 0          # layout of another sequence
    assert runtime.last_block_window(None, 5000) == 0
    gap = SimpleNamespace(seq_len=5000, segments=[(0, 700, "text"), (700, 3900, "video"), (4000, 5000, "audio")])
    assert runtime.last_block_window({"layout": gap}, 5000) == 0          # spans not contiguous
    one = SimpleNamespace(seq_len=5000, segments=[(0, 700, "text"), (700, 5000, "video")])
    assert runtime.last_block_window({"layout": one}, 5000) == 0          # the reference needs two spans


def test_qkv_op_rejects_wrong_geometry_before_any_launch():
    """ops/qkv.py:24-40 of the reference: the H3 geometry, the RoPE layout and the
    operand dtypes are checked first, with the reference's messages."""
    import torch
    from h3_speedkit.ops.qkv import QKV
    op = QKV()
    m = 4
    q = torch.zeros((m, 5376), dtype=torch.int8)
    w = torch.zeros((21504, 5376), dtype=torch.int8)
    xs, ws = torch.zeros((m, 1)), torch.zeros((21504, 1))
    rope = torch.zeros((1, m, 1, 48, 2, 2), dtype=torch.bfloat16)
    qw = kw = torch.zeros((128,), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="H3 56 x 128, hidden=5376"):
        op(q[:, :5120], w, xs, ws, rope, qw, kw, 1e-6)
    with pytest.raises(ValueError, match="pinned partial split-half RoPE layout"):
        op(q, w, xs, ws, rope.view(1, m, 1, 96, 2), qw, kw, 1e-6)
    with pytest.raises(ValueError, match="does not match the CUDA ABI"):
        op(q, w, xs.double(), ws, rope, qw, kw, 1e-6)
    with pytest.raises(ValueError, match="contiguous and on one CUDA device"):
        op(q, w, xs, ws, rope, qw, kw, 1e-6)
