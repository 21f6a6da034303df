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
import ctypes as ct

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


def _h3_block_ns(bw, qw, kw):
    from types import SimpleNamespace as NS

    def linear(w, s):
        return NS(weight=w, weight_int8=w, weight_scale=s)

    return NS(adaln_proj=lambda t: (bw.shift_msa, bw.scale_msa, bw.gate_msa, bw.shift_mlp, bw.scale_mlp,
                                    bw.gate_mlp),
              norm1=NS(weight=bw.norm1, eps=1e-6), norm2=NS(weight=bw.norm2, eps=1e-6),
              attn=NS(qkv_proj=linear(bw.qkv, bw.qkv_s), out_proj=linear(bw.out, bw.out_s),
                      q_norm=NS(weight=qw, eps=1e-6), k_norm=NS(weight=kw, eps=1e-6)),
              mlp=NS(fc1=linear(bw.fc1, bw.fc1_s), fc2=linear(bw.fc2, bw.fc2_s)))


def _reference_block(x, bw, qw, kw, rope, rows, skip):
    """runtime.py:126-164 of the reference as a chain of its own kernels (compiled
    from its sources): the K=5376 prologue, the sample gather, the K anchor
    detector, the fused QKV kernel r84_kfourwarp.cu, the INT8 attention
    dense_ring.cu, the register ConvRot quantiser, gate.cu and fc1.cu, the
    Kitchen SwiGLU quantiser.  Two steps have no C kernel in the reference and
    come from this library, pinned elsewhere: the K-only sample projection and
    the V quantiser (Triton in the reference)."""
    from h3_speedkit import _lib
    lib = _lib.load()
    dev, m = x.device, x.shape[0]
    st = torch.cuda.current_stream().cuda_stream
    q, qs = ref_gpu.norm_quant(x, bw.norm1, bw.shift_msa, bw.scale_msa, rows, 1e-6)
    sq, sx, sr = ref_gpu.sample_gather(q, qs, rope.view(m, 192))
    sd = torch.empty((3, 56, 9, 128), dtype=torch.bfloat16, device=dev)
    assert lib.h3_sample_konly_ex(sq.data_ptr(), bw.qkv.data_ptr(), sx.data_ptr(), bw.qkv_s.data_ptr(),
                                  sd.data_ptr(), sr.data_ptr(), qw.data_ptr(), kw.data_ptr(),
                                  ct.c_float(1e-6), 9, 56, 5376, None, st) == 1
    sk = sd[1].contiguous()
    anchors = ref_gpu.sample_anchor(sk)
    t = ref_gpu.qkv_quant_kv(q, bw.qkv, qs, bw.qkv_s, rope, qw, kw, 1e-6, sk, anchors)
    parts = (m + 127) // 128
    vi = torch.empty((56 * 128, parts * 128), dtype=torch.int8, device=dev)
    vs = torch.empty((56 * 128,), dtype=torch.float32, device=dev)
    vinv = torch.empty_like(vs)
    assert lib.h3_quant_v(t["vp"].data_ptr(), t["d"][2].data_ptr(), vi.data_ptr(), vs.data_ptr(),
                          vinv.data_ptr(), m, 56, st) == 1
    o = ref_gpu.dense(t["qi"].view(1, 56, m, 128), t["ki"].view(1, 56, m, 128), vi,
                      t["qs"].view(1, 56, parts * 32), t["ks"].view(1, 56, parts * 4), vs, 128 ** -0.5,
                      layout="bshd", start=skip // 128)
    attn = o.transpose(1, 2).reshape(m, 7168)
    aq, asc, _ = ref_gpu.convrot_register(attn, 0)
    w = slice(skip, None)
    ref_gpu.int8_gate(aq[w], bw.out, asc.view(-1)[w], bw.out_s, bw.gate_msa, rows[w], x[w], out=x[w])
    q, qs = ref_gpu.norm_quant(x, bw.norm2, bw.shift_mlp, bw.scale_mlp, rows, 1e-6)
    hidden = torch.zeros((m, bw.fc1.shape[0]), dtype=torch.bfloat16, device=dev)
    hidden[w] = ref_gpu.int8(q[w].contiguous(), bw.fc1, qs.view(-1)[w].contiguous(), bw.fc1_s)
    hq, hs = ref_gpu.kitchen_quant(hidden, 2)
    ref_gpu.int8_gate(hq[w], bw.fc2, hs.view(-1)[w], bw.fc2_s, bw.gate_mlp, rows[w], x[w], out=x[w])
    return x


@pytest.mark.parametrize("skip", [0, 256])
def test_runtime_block_with_int8_attention_equals_reference_chain(device, skip):
    """Backend.block(attention="int8") -- the reference's whole block, attention
    included -- at the H3 geometry (hidden 5376, 56 heads, SwiGLU MLP, two adaLN
    table rows), with and without the last-block window: bit for bit the chain
    of the reference's own kernels."""
    from h3_speedkit import synthetic
    from h3_speedkit.runtime import Backend
    for name in ("ref_dense.so", "ref_qkv.so", "ref_gather.so", "ref_anchor.so", "ref_fc1.so", "ref_gate.so",
                 "ref_kitchen.so", "ref_convrot.so", "ref_norm_k5376.so"):
        if not ref_gpu.available(name):
            pytest.fail(f"oracle/_ref/{name} is missing: build it with oracle/build.py")
    m = 512
    bw = synthetic.h3_block(0, tables=2, device=device)
    g = torch.Generator(device=device).manual_seed(77)
    ang = torch.rand((m, 48), generator=g, device=device) * 6.283
    rope = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).reshape(1, m, 1, 48, 2, 2)
    rope = rope.to(torch.bfloat16)
    qw = (torch.rand((128,), generator=g, device=device) + 0.5).to(torch.bfloat16)
    kw = (torch.rand((128,), generator=g, device=device) + 0.5).to(torch.bfloat16)
    x0 = synthetic.cfg5_tokens(m, 5376, device=device)
    rows = (torch.arange(m, device=device) % 2).to(torch.int32)
    ours = x0.clone()
    Backend().block(_h3_block_ns(bw, qw, kw), ours, None, None, rope, rows=rows, skip=skip, attention="int8",
                    mlp_act="swiglu")
    ref = _reference_block(x0.clone(), bw, qw, kw, rope, rows, skip)
    torch.cuda.synchronize()
    assert torch.equal(ours, ref)


@pytest.mark.parametrize("batch,sq,sk,heads,kv_heads", [(2, 300, 700, 4, 2), (3, 129, 129, 2, 2),
                                                         (2, 640, 128, 2, 1)])
def test_attention_batches_and_unequal_lengths_equal_reference(device, batch, sq, sk, heads, kv_heads):
    """Batch > 1 and query length != key length (the ABI's separate qo_len /
    kv_len and batch strides): the same bits as the reference kernel."""
    _need()
    g = torch.Generator().manual_seed(batch * 1000 + sq + sk)
    pq, pk = (sq + 127) // 128, (sk + 127) // 128
    q = torch.randint(-127, 128, (batch, heads, sq, 128), generator=g, dtype=torch.int8)
    k = torch.randint(-127, 128, (batch, kv_heads, sk, 128), generator=g, dtype=torch.int8)
    v = torch.randint(-127, 128, (batch * kv_heads * 128, pk * 128), generator=g, dtype=torch.int8)
    qs = torch.rand((batch, heads, pq * 32), generator=g) * 0.02 + 0.001
    ks = torch.rand((batch, kv_heads, pk * 4), generator=g) * 0.02 + 0.001
    vs = torch.rand((batch * kv_heads * 128,), generator=g) * 0.01 + 0.0005
    packed = PrequantizedInt8Attention(
        q=q.to(device), k=k.to(device), v=v.to(device), q_scale=qs.to(device), k_scale=ks.to(device),
        v_scale=vs.to(device), original_head_dim=128, input_dtype=torch.bfloat16, attention_scale=128 ** -0.5,
        cta_k=128, attn_mask=None)
    for layout in ("bshd", "bhsd"):
        _compare(packed, layout)
