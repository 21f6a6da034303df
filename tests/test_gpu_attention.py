"""GPU parity of the INT8 attention (h3_dense_launch_window) against the
reference's own kernel.

oracle/build.py compiles the reference's kernels/dense/dense_ring.cu (the
SageAttention-derived mma.sync kernel, variant 8102) for sm_100a from its
sources; here it runs on the same operands as this build's tcgen05 kernel and
the BF16 outputs must be the same bits.  The operands come from this build's QKV
op (pinned to the reference's r84_kfourwarp.cu elsewhere) on seeded projections
-- Q/K codes with their per-group scales, V codes channel-major in the
reference's key permutation -- and, for the corner cases, from seeded random
codes and scales.
"""
import pytest
import torch

from h3_speedkit.ops.dense import DenseLibrary, allocate_output
from h3_speedkit.ops.qkv import QKV, PrequantizedInt8Attention
from oracle import ref_gpu

pytestmark = pytest.mark.gpu


def _need():
    if not ref_gpu.available("ref_dense.so"):
        pytest.fail("oracle/_ref/ref_dense.so is missing: build it with oracle/build.py")


def _from_qkv(m, heads, hidden, seed, device):
    """Attention operands of a seeded QKV projection through this build's QKV op."""
    g = torch.Generator().manual_seed(seed)
    n = 3 * heads * 128
    q = torch.randint(-127, 128, (m, hidden), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, hidden), generator=g, dtype=torch.int8)
    xs = torch.rand((m, 1), generator=g) * 0.009 + 0.001
    ws = torch.rand((n, 1), generator=g) * 0.0045 + 0.0005
    ang = torch.rand((m, 48), generator=g) * 6.283
    rope = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).reshape(1, m, 1, 48, 2, 2)
    qw = (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16)
    kw = (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16)
    args = [t.to(device) for t in (q, w, xs.float(), ws.float(), rope.to(torch.bfloat16), qw, kw)]
    out = QKV().run(*args, 1e-6, heads=heads)
    parts = (m + 127) // 128
    return PrequantizedInt8Attention(
        q=out["qi"].view(1, heads, m, 128), k=out["ki"].view(1, heads, m, 128), v=out["vi"],
        q_scale=out["qs"].view(1, heads, parts * 32), k_scale=out["ks"].view(1, heads, parts * 4),
        v_scale=out["vs"], original_head_dim=128, input_dtype=torch.bfloat16, attention_scale=128 ** -0.5,
        cta_k=128, attn_mask=None)


def _random(m, heads, kv_heads, seed, device, spread=1.0):
    """Seeded random codes and scales in the same layouts (spread scales the
    Q and K scales: larger scores make sharper softmax rows)."""
    g = torch.Generator().manual_seed(seed)
    parts = (m + 127) // 128
    q = torch.randint(-127, 128, (1, heads, m, 128), generator=g, dtype=torch.int8)
    k = torch.randint(-127, 128, (1, kv_heads, m, 128), generator=g, dtype=torch.int8)
    v = torch.randint(-127, 128, (kv_heads * 128, parts * 128), generator=g, dtype=torch.int8)
    qs = (torch.rand((1, heads, parts * 32), generator=g) * 0.02 + 0.001) * spread
    ks = (torch.rand((1, kv_heads, parts * 4), generator=g) * 0.02 + 0.001) * spread
    vs = torch.rand((kv_heads * 128,), generator=g) * 0.01 + 0.0005
    return PrequantizedInt8Attention(
        q=q.to(device), k=k.to(device), v=v.to(device), q_scale=qs.to(device), k_scale=ks.to(device),
        v_scale=vs.to(device), original_head_dim=128, input_dtype=torch.bfloat16, attention_scale=128 ** -0.5,
        cta_k=128, attn_mask=None)


def _compare(packed, layout="bshd", start=0):
    out = allocate_output(packed, layout)
    DenseLibrary().bind(packed, out, start=start)()
    ref = ref_gpu.dense(packed.q, packed.k, packed.v, packed.q_scale, packed.k_scale, packed.v_scale,
                        packed.attention_scale, layout=layout, start=start)
    torch.cuda.synchronize()
    a, b = out.contiguous().view(torch.int16), ref.contiguous().view(torch.int16)
    if start:
        a, b = a[:, :, start * 128:], b[:, :, start * 128:]
    diff = int((a != b).sum())
    assert diff == 0, f"{diff} of {a.numel()} outputs differ"
    return out


@pytest.mark.parametrize("m,heads,hidden", [(1000, 2, 256), (300, 4, 512), (129, 2, 256), (128, 2, 256),
                                            (1, 2, 256), (2048, 56, 5376)])
def test_attention_on_qkv_operands_equals_reference(device, m, heads, hidden):
    """The QKV op's outputs fed to both attention kernels: one block and many,
    ragged last blocks, a single token, the H3 geometry (56 heads)."""
    _need()
    _compare(_from_qkv(m, heads, hidden, 13 * m + heads, device))


@pytest.mark.parametrize("m,heads,kv_heads,spread", [(777, 4, 4, 1.0), (640, 4, 2, 1.0), (300, 2, 2, 8.0),
                                                     (256, 2, 1, 0.05), (4096 + 3, 2, 2, 1.0)])
def test_attention_on_random_codes_equals_reference(device, m, heads, kv_heads, spread):
    """Random codes and scales: grouped KV heads, sharp (large scores) and flat
    (tiny scores) softmax rows, exact multiples of the block and ragged ends."""
    _need()
    _compare(_random(m, heads, kv_heads, 7 * m + heads + kv_heads, device, spread))


@pytest.mark.parametrize("layout,start", [("bhsd", 0), ("bshd", 2), ("bhsd", 3)])
def test_attention_layouts_and_row_window(device, layout, start):
    """BHSD and BSHD output storage; a row window that starts at query block
    `start` (rows before it are zero, the last-block window of runtime.py:151-155)."""
    _need()
    packed = _random(700, 2, 2, 91 + start, device)
    out = _compare(packed, layout, start)
    if start:
        assert not out[:, :, :start * 128].float().abs().any()


def test_attention_rejects_bad_layouts_before_launch(device):
    import dataclasses
    packed = _random(300, 2, 2, 5, device)
    lib = DenseLibrary()
    with pytest.raises(ValueError, match="Kitchen's"):
        lib.bind(dataclasses.replace(packed, v=packed.v[:, :256].contiguous()), allocate_output(packed))
    padded = torch.empty((1, 2, 400, 128), dtype=torch.bfloat16, device=device)[:, :, :300]
    with pytest.raises(ValueError, match="BHSD or BSHD"):
        lib.bind(packed, padded)
