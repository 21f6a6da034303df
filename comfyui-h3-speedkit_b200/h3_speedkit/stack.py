"""The quantized DiT-block linear chain and its token-sharded block stack.

One block (the linear path of ``Backend.block``, runtime.py:126-164 of H3
SpeedKit, with attention replaced by an identity passthrough of V):

    q, qs   = prologue(x; norm1, shift_msa, scale_msa)        fused RMSNorm/adaLN/ConvRot/INT8
    qkv     = bf(dequant(q . Wqkv^T))                           INT8 GEMM, N = 3D
    aq, as  = convrot_quant(qkv[:, 2D:3D])                      identity attention: V
    x       = bf(fmaf(bf(dequant(aq . Wout^T)), gate_msa, x))   outproj gate-residual, in place
    q, qs   = prologue(x; norm2, shift_mlp, scale_mlp)
    h       = bf(gelu_tanh(bf(dequant(q . Wfc1^T))))            FC1 + GELU epilogue
    hq, hs  = convrot_quant(h)                                  ACT none (GELU already applied)

Both quantisers after a GEMM run split: the GEMM's epilogue also rotates each
256-column group it feeds to the quantiser (all of h; the V third of qkv) and
keeps each row's max |rotated value|, then a codes pass over the rotated rows
writes the same codes and scales bit for bit.
    x       = bf(fmaf(bf(dequant(hq . Wfc2^T)), gate_mlp, x))   FC2 gate-residual, in place

Every op is row-local, so a contiguous token shard gives bit-identical rows on
any number of GPUs.  ``ShardedStack`` splits the tokens across the ranks of a
torch.distributed process group (weights replicated), runs the blocks with no
collective, and gathers the final BF16 rows with one all_gather_into_tensor.

``BlockPlan`` binds one block's launches to preallocated buffers once and then
replays them through the C-ABI with fixed pointers, so a step is a short list of
ctypes calls on the current stream (and can be captured in a CUDA graph).
"""
from __future__ import annotations

import weakref

from dataclasses import dataclass

import torch

from . import _lib
from .synthetic import BlockWeights

ACT_NONE, ACT_SWIGLU = 0, 2
EPI_DEQUANT, EPI_GELU = 0, 1
GEMM_NAMES = ("qkv", "outproj", "fc1", "fc2")


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous token block of `rank`: rows [start, stop).  Ranks get
    ceil(total/world) rows except the tail, which may be shorter or empty."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("invalid rank/world")
    per = -(-total // world)
    start = min(total, rank * per)
    return start, min(total, start + per)


def _round_up(v: int, unit: int) -> int:
    return -(-v // unit) * unit


def uniform_chunks(per: int, chunks: int) -> list[tuple[int, int]]:
    """``chunks`` contiguous row ranges of (nearly) equal size covering [0, per)."""
    step = -(-per // max(1, chunks))
    return [(c0, min(per, c0 + step)) for c0 in range(0, per, step)]


def chunk_schedule(per: int, world: int, unit: int = 128, min_rows: int = 1024) -> list[tuple[int, int]]:
    """Row ranges of the end-to-end pipeline over one rank's padded shard of
    ``per`` rows (identical on every rank).

    The copy in of the first chunk and the copy out of the last chunk are the
    only transfers not hidden behind compute, so both end chunks are small
    (per/16 rows, at least ``min_rows``; smaller chunks lose more to kernel ramp
    and tail than they save in copy time).  Chunks grow 4x at the head (a chunk's
    host->device copy takes about a tenth of its compute) and shrink at the tail
    by a factor that follows the device->host share: rank 0 copies out the rows
    of all ``world`` ranks, about 0.1 x world of a chunk's compute, so each tail
    chunk is at least that fraction of the one before it and the copy-out queue
    never grows.  Middle chunks are per/4 rows.  Sizes are multiples of ``unit``
    (one remainder chunk in the middle takes the rest)."""
    if per < 8 * min_rows:
        return uniform_chunks(per, max(1, min(4, per // 2048)))
    big = _round_up(per // 4, unit)
    small = max(min_rows, _round_up(per // 16, unit))
    down = min(0.8, max(0.25, 0.1 * world))
    head, s = [], small
    while s < big:
        head.append(s)
        s = _round_up(4 * s, unit)
    tail, s = [], small
    while s < big:
        tail.append(s)
        s = _round_up(int(s / down), unit)
    while sum(head) + sum(tail) > per and len(head) + len(tail) > 2:
        (head if len(head) > 1 else tail).pop()   # drop the largest ramp chunk
    mid = per - sum(head) - sum(tail)
    if mid < 0:
        return uniform_chunks(per, 4)
    middle = []
    if 0 < mid < small and len(head) > 1:
        head[-1] += mid   # a small remainder joins the largest head chunk
        mid = 0
    if mid:
        n_mid = -(-mid // big)
        part = _round_up(-(-mid // n_mid), unit)
        while mid > 0:
            middle.append(min(part, mid))
            mid -= middle[-1]
    bounds, c0 = [], 0
    for size in head + middle + tail[::-1]:
        bounds.append((c0, c0 + size))
        c0 += size
    return bounds


def shared_host_output(rows: int, d: int, dtype=torch.bfloat16, group=None,
                       directory: str = "/dev/shm") -> torch.Tensor | None:
    """A pinned host tensor [rows, d] that every rank of ``group`` (one node)
    maps: a POSIX shared-memory file under ``directory``, mapped MAP_SHARED in
    each process and page-locked there with cudaHostRegister, so that every
    rank's device-to-host copies land in the one buffer over the rank's own PCIe
    link (``ShardedStack.forward_host(..., shared_out=True)``).  The file is
    unlinked once every rank has mapped it.  Returns None on every rank when the
    file system lacks the room or a process cannot page-lock the mapping."""
    import os
    import uuid

    import torch.distributed as dist
    multi = dist.is_initialized() and dist.get_world_size(group) > 1
    rank = dist.get_rank(group) if multi else 0
    nbytes = rows * d * torch.empty((), dtype=dtype).element_size()
    path = ""
    if rank == 0:
        try:
            st = os.statvfs(directory)
            if st.f_bavail * st.f_frsize >= nbytes + (64 << 20):
                path = os.path.join(directory, f"h3sk_out_{os.getpid()}_{uuid.uuid4().hex[:12]}")
        except OSError:
            path = ""
    if multi:
        box = [path]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        path = box[0]
    if not path:
        return None
    def mapping():
        try:
            return torch.from_file(path, shared=True, size=nbytes, dtype=torch.uint8)
        except Exception:   # e.g. no room in the file system
            return None

    # every rank takes the same collective steps on every path
    base = mapping() if rank == 0 else None
    if multi:
        dist.barrier(group=group)   # the file exists (or rank 0 failed) before the others map it
    if rank != 0:
        base = mapping()
    ok = 0
    if base is not None:
        try:
            rc = torch.cuda.cudart().cudaHostRegister(base.data_ptr(), nbytes, 0)
            ok = 1 if int(rc) == 0 else 0
            if not ok:
                torch.cuda.cudart().cudaGetLastError()   # clear the failed call's error state
        except Exception:   # no CUDA runtime: the buffer cannot be page-locked
            ok = 0
    if multi:
        on_gpu = dist.get_backend(group) == "nccl"
        flag = torch.tensor([ok], dtype=torch.int32, device=torch.cuda.current_device() if on_gpu else "cpu")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        all_ok = bool(flag.item())
        dist.barrier(group=group)
    else:
        all_ok = bool(ok)
    if rank == 0:
        try:
            os.unlink(path)
        except OSError:
            pass
    if not all_ok:
        if ok and base is not None:
            torch.cuda.cudart().cudaHostUnregister(base.data_ptr())
        return None
    out = base.view(dtype).view(rows, d)
    # Page-locking lasts as long as the returned tensor: when it is collected the
    # registration is removed before the mapping itself can go (the finalizer holds
    # the mapping until then).  Views taken from `out` that outlive it keep the
    # memory mapped but no longer page-locked.
    weakref.finalize(out, _host_unregister, base.data_ptr(), base)
    return out


def _host_unregister(ptr: int, _mapping) -> None:
    try:
        torch.cuda.cudart().cudaHostUnregister(ptr)
    except Exception:   # interpreter shutdown: the process exit releases it
        pass


def gather_shards(send: torch.Tensor, out: torch.Tensor, total: int, group=None) -> torch.Tensor:
    """Assemble the token-sharded output: every rank contributes its padded shard
    ``send`` [ceil(total/world), D]; ``out`` [world * ceil(total/world), D]
    receives all of them in rank order (one all_gather_into_tensor); the first
    ``total`` rows are returned."""
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return send[:total]
    dist.all_gather_into_tensor(out, send, group=group)
    return out[:total]


@dataclass
class Workspace:
    """Per-shard activation buffers, sized once for m rows."""
    q: torch.Tensor
    qs: torch.Tensor
    qkv: torch.Tensor
    aq: torch.Tensor
    as_: torch.Tensor
    h: torch.Tensor
    hq: torch.Tensor
    hs: torch.Tensor
    hmax: torch.Tensor   # int32 [m]: FP32 bits of each row's max |rotated h| (rotation in FC1's epilogue)
    vmax: torch.Tensor   # int32 [m]: the same for the rotated V third of qkv (rotation in the QKV epilogue)

    @classmethod
    def allocate(cls, m: int, d: int, ffn: int, device, *, attn: int | None = None,
                 fc1_n: int | None = None) -> "Workspace":
        e = dict(device=device)
        attn = d if attn is None else attn
        fc1_n = ffn if fc1_n is None else fc1_n
        return cls(q=torch.empty((m, d), dtype=torch.int8, **e), qs=torch.empty((m, 1), dtype=torch.float32, **e),
                   qkv=torch.empty((m, 3 * attn), dtype=torch.bfloat16, **e),
                   aq=torch.empty((m, attn), dtype=torch.int8, **e),
                   as_=torch.empty((m, 1), dtype=torch.float32, **e),
                   h=torch.empty((m, fc1_n), dtype=torch.bfloat16, **e),
                   hq=torch.empty((m, ffn), dtype=torch.int8, **e), hs=torch.empty((m, 1), dtype=torch.float32, **e),
                   hmax=torch.empty((m,), dtype=torch.int32, **e), vmax=torch.empty((m,), dtype=torch.int32, **e))

    @classmethod
    def for_block(cls, m: int, weights: BlockWeights, device) -> "Workspace":
        g = geometry(weights)
        return cls.allocate(m, g["d"], g["ffn"], device, attn=g["attn"], fc1_n=g["fc1_n"])


def geometry(weights: BlockWeights) -> dict:
    """Block geometry from the weight shapes: width d, attention width (QKV N / 3),
    FFN width (FC2 K), FC1 N, and whether the MLP is SwiGLU (FC1 N = 2 FFN)."""
    d = weights.norm1.shape[0]
    attn = weights.qkv.shape[0] // 3
    ffn = weights.fc2.shape[1]
    fc1_n = weights.fc1.shape[0]
    if (weights.qkv.shape != (3 * attn, d) or weights.out.shape != (d, attn) or weights.fc1.shape[1] != d
            or weights.fc2.shape[0] != d or fc1_n not in (ffn, 2 * ffn)):
        raise ValueError("inconsistent block weight shapes")
    return {"d": d, "attn": attn, "ffn": ffn, "fc1_n": fc1_n, "swiglu": fc1_n == 2 * ffn}


class BlockPlan:
    """One block's launches, bound to fixed buffers.

    ``x`` is updated in place.  ``rows`` maps each token to a row of the adaLN /
    gate tables.  ``skip`` is the reference's last-block row window
    (runtime.py:117-160, applied to block 49 only, runtime.py:296): rows
    [0, skip) keep their residual -- no outproj, FC1 or FC2 work for them --
    while QKV still covers every row (attention reads all keys and values).
    With identity attention the V quantiser and the second prologue also start
    at ``skip``: their rows below it feed nothing.  Nothing is allocated when
    the plan runs.

    ``epilogue_rotation``: the QKV GEMM's epilogue runs the V quantiser's
    ConvRot256 on the V third and, in GELU blocks, FC1's epilogue runs the
    FC2-input quantiser's on all of h, each keeping the rows' max |rotated value|
    (``h3_int8_rot``); a light pass then writes the codes and scales
    (``h3_convrot_codes``).  Same aq, as, hq, hs bit for bit as the GEMMs
    followed by the full quantisers (False), and faster: the rotations run in
    the GEMMs' epilogue warps while the tensor cores work.
    """

    def __init__(self, weights: BlockWeights, x: torch.Tensor, rows: torch.Tensor, ws: Workspace,
                 eps: float = 1e-6, skip: int = 0, epilogue_rotation: bool = True):
        self.lib = _lib.load()
        m, d = x.shape
        g = geometry(weights)
        attn, ffn, n1 = g["attn"], g["ffn"], g["fc1_n"]
        if g["d"] != d:
            raise ValueError("block weights do not match the activation width")
        if m < 1:
            raise ValueError("empty shard")
        if not 0 <= skip <= m:
            raise ValueError("row window outside the shard")
        if ws.qkv.shape[1] != 3 * attn or ws.h.shape[1] != n1 or ws.hq.shape[1] != ffn or ws.aq.shape[1] != attn:
            raise ValueError("workspace does not match the block geometry")
        self.keep = (weights, x, rows, ws)   # owners of every pointer below
        self.skip = skip
        lib = self.lib
        w = weights
        tdt = int(w.shift_msa.dtype == torch.bfloat16)
        fc1_epi, mlp_act = (EPI_DEQUANT, ACT_SWIGLU) if g["swiglu"] else (EPI_GELU, ACT_NONE)
        s, n = skip, m - skip   # the window: rows [s, m)

        def P(t, row=0):
            """Address of row `row` of a 2-D tensor (or element `row` of a 1-D one)."""
            return t.data_ptr() + row * t.stride(0) * t.element_size()

        calls = [
            ("prologue", lib.h3_norm_quant_run_t,
             (P(x), P(w.norm1), P(w.shift_msa), P(w.scale_msa), P(rows), P(ws.q), P(ws.qs), None, None, None,
              m, d, w.shift_msa.shape[0], x.stride(0), w.shift_msa.stride(0), w.scale_msa.stride(0), float(eps),
              tdt, 0)),
        ]
        # qkv's V third (columns [2 attn, 3 attn)), the identity attention's output
        if epilogue_rotation:
            calls.append(("qkv", lib.h3_int8_rot,
                          (P(ws.q), P(w.qkv), P(ws.qs), P(w.qkv_s), None, P(ws.qkv), P(ws.vmax), m, 3 * attn, d,
                           3 * attn, 0, 2 * attn)))
            quant_v = ("quant_v", lib.h3_convrot_codes,
                       (P(ws.qkv, s) + 2 * attn * 2, 3 * attn, P(ws.vmax, s), P(ws.aq, s), P(ws.as_, s), n, attn))
        else:
            calls.append(("qkv", lib.h3_int8_ex,
                          (P(ws.q), P(w.qkv), P(ws.qs), P(w.qkv_s), None, P(ws.qkv), m, 3 * attn, d, 3 * attn,
                           EPI_DEQUANT)))
            quant_v = ("quant_v", lib.h3_convrot_quant_act,
                       (P(ws.qkv, s) + 2 * attn * 2, 3 * attn, P(ws.aq, s), P(ws.as_, s), n, attn, ACT_NONE))
        if n:
            calls += [
                quant_v,
                ("outproj", lib.h3_int8_gate,
                 (P(ws.aq, s), P(w.out), P(ws.as_, s), P(w.out_s), P(x, s), P(w.gate_msa), P(rows, s), P(x, s), n, d,
                  attn, 13)),
                ("prologue", lib.h3_norm_quant_run_t,
                 (P(x, s), P(w.norm2), P(w.shift_mlp), P(w.scale_mlp), P(rows, s), P(ws.q, s), P(ws.qs, s), None,
                  None, None, n, d, w.shift_mlp.shape[0], x.stride(0), w.shift_mlp.stride(0),
                  w.scale_mlp.stride(0), float(eps), tdt, 0)),
            ]
            if epilogue_rotation and not g["swiglu"]:
                calls += [
                    ("fc1", lib.h3_int8_gelu_rot,
                     (P(ws.q, s), P(w.fc1), P(ws.qs, s), P(w.fc1_s), None, P(ws.h, s), P(ws.hmax, s), n, n1, d,
                      n1)),
                    ("quant_h", lib.h3_convrot_codes,
                     (P(ws.h, s), n1, P(ws.hmax, s), P(ws.hq, s), P(ws.hs, s), n, ffn)),
                ]
            else:
                calls += [
                    ("fc1", lib.h3_int8_ex,
                     (P(ws.q, s), P(w.fc1), P(ws.qs, s), P(w.fc1_s), None, P(ws.h, s), n, n1, d, n1, fc1_epi)),
                    ("quant_h", lib.h3_convrot_quant_act,
                     (P(ws.h, s), n1, P(ws.hq, s), P(ws.hs, s), n, ffn, mlp_act)),
                ]
            calls += [
                ("fc2", lib.h3_int8_gate,
                 (P(ws.hq, s), P(w.fc2), P(ws.hs, s), P(w.fc2_s), P(x, s), P(w.gate_mlp), P(rows, s), P(x, s), n, d,
                  ffn, 13)),
            ]
        self.calls = calls

    def launch(self, stream: int, events=None) -> None:
        """Enqueue the eight launches on `stream`.  With `events` (a dict of
        name -> list of (start, end) CUDA event pairs) each launch is bracketed."""
        for name, fn, args in self.calls:
            if events is not None:
                start = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
                start.record()
            rc = fn(*args, stream)
            if name in GEMM_NAMES:
                _lib.check_int8(rc)          # GEMM entry points return 1 on success
            elif rc != 0:                    # the others return a cudaError_t
                raise RuntimeError(f"{name} launch failed with CUDA error {rc}")
            if events is not None:
                end.record()
                events.setdefault(name, []).append((start, end))

    @staticmethod
    def gemm_ops(m: int, d: int, ffn: int, attn: int | None = None, fc1_n: int | None = None) -> dict:
        attn = d if attn is None else attn
        fc1_n = ffn if fc1_n is None else fc1_n
        return {"qkv": 2 * m * 3 * attn * d, "outproj": 2 * m * d * attn, "fc1": 2 * m * fc1_n * d,
                "fc2": 2 * m * d * ffn}


def block_ops_per_token(d: int = 4096, ffn: int = 16384) -> int:
    """INT8 ops per token per block: 2*D*(3D + D + FFN) + 2*FFN*D."""
    return 2 * d * (3 * d + d + ffn) + 2 * ffn * d


class LocalStack:
    """All blocks over one contiguous shard of tokens, on the current device."""

    def __init__(self, blocks: list[BlockWeights], x: torch.Tensor, rows: torch.Tensor, eps: float = 1e-6,
                 ws: Workspace | None = None, skip: int = 0, epilogue_rotation: bool = True):
        """``skip``: the last block's row window (rows [0, skip) of this shard keep
        the residual the previous blocks left; see BlockPlan).  ``epilogue_rotation``:
        see BlockPlan."""
        m, d = x.shape
        self.x, self.rows = x, rows
        if ws is not None and ws.q.shape[0] < m:
            raise ValueError("shared workspace too small for this shard")
        self.ws = ws if ws is not None else Workspace.for_block(m, blocks[0], x.device)
        self.plans = [BlockPlan(b, x, rows, self.ws, eps, skip=skip if i == len(blocks) - 1 else 0,
                                epilogue_rotation=epilogue_rotation)
                      for i, b in enumerate(blocks)]
        self.graph = None

    @property
    def launches_per_step(self) -> int:
        return sum(len(plan.calls) for plan in self.plans)

    def run(self, events=None) -> torch.Tensor:
        if self.graph is not None and events is None:
            self.graph.replay()
            return self.x
        stream = torch.cuda.current_stream(self.x.device).cuda_stream
        for plan in self.plans:
            plan.launch(stream, events)
        return self.x

    def capture(self) -> None:
        """Capture the whole stack as one CUDA graph (fixed buffers, no host work per step)."""
        torch.cuda.synchronize(self.x.device)
        stream = torch.cuda.Stream(self.x.device)
        stream.wait_stream(torch.cuda.current_stream(self.x.device))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph, stream=stream):
                self.run()
        torch.cuda.current_stream(self.x.device).wait_stream(stream)
        self.graph = graph


class ShardedStack:
    """Token-sharded block stack: rank r owns rows shard_bounds(M, world, r),
    weights are replicated, one all_gather_into_tensor assembles the output.

    The shard lives in ``self.send`` (padded to ceil(M/world) rows); the blocks
    update it in place and the same buffer feeds the all-gather, so no copy
    sits between the last block and the collective.
    """

    def __init__(self, blocks, rows_shard: torch.Tensor, total_rows: int, d: int, device, group=None,
                 eps: float = 1e-6, dtype=torch.bfloat16, skip: int = 0):
        """``skip``: the last block's row window as a global row index (the first
        target token rounded down to 128 in the reference, runtime.py:207); each
        rank applies the part that falls in its shard."""
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.start, self.stop = shard_bounds(total_rows, self.world, self.rank)
        self.rows_local = self.stop - self.start
        if rows_shard.shape[0] != self.rows_local:
            raise ValueError(f"rank {self.rank} expects {self.rows_local} table rows, got {rows_shard.shape[0]}")
        self.total = total_rows
        self.per = -(-total_rows // self.world)
        self.send = torch.zeros((self.per, d), dtype=dtype, device=device)
        self.out = torch.empty((self.per * self.world, d), dtype=dtype, device=device)
        self.x = self.send[: self.rows_local]
        if not 0 <= skip <= total_rows:
            raise ValueError("row window outside the token range")
        self.skip_local = min(max(skip - self.start, 0), self.rows_local)
        self.local = LocalStack(blocks, self.x, rows_shard, eps, skip=self.skip_local) if self.rows_local else None
        self._blocks, self._rows, self._eps = blocks, rows_shard, eps

    @property
    def launches_per_step(self) -> int:
        return self.local.launches_per_step if self.local is not None else 0

    def load(self, x_shard: torch.Tensor, non_blocking: bool = True) -> None:
        """Copy this rank's input rows (device or pinned host) into the shard buffer."""
        if x_shard.shape != self.x.shape:
            raise ValueError(f"expected input shard {tuple(self.x.shape)}, got {tuple(x_shard.shape)}")
        self.x.copy_(x_shard, non_blocking=non_blocking)

    def forward_local(self, events=None) -> None:
        if self.local is not None:
            self.local.run(events)

    def gather(self) -> torch.Tensor:
        return gather_shards(self.send, self.out, self.total, self.group)

    def forward(self, events=None) -> torch.Tensor:
        self.forward_local(events)
        return self.gather()

    # ---- end to end from pinned host memory, copies overlapped with compute -------
    def _chunking(self, chunks: int | None, schedule_world: int | None = None):
        """Chunk boundaries over the padded shard (identical on every rank, so every
        rank issues the same collectives) and one LocalStack per chunk sharing one
        workspace sized for the largest chunk.  ``chunks=None`` takes
        ``chunk_schedule`` (small end chunks, ramped tail); an int gives that many
        equal chunks."""
        schedule_world = self.world if schedule_world is None else schedule_world
        key = ("chunks", chunks, schedule_world)
        cached = getattr(self, "_chunk_cache", None)
        if cached is not None and cached[0] == key:
            return cached[1]
        bounds = chunk_schedule(self.per, schedule_world) if chunks is None else uniform_chunks(self.per, chunks)
        step = max(c1 - c0 for c0, c1 in bounds)
        stacks = []
        ws = None
        if self.local is not None:
            ws = Workspace.for_block(step, self._blocks[0], self.x.device)
        for c0, c1 in bounds:
            hi = min(c1, self.rows_local)
            if self.local is not None and hi > c0:
                window = min(max(self.skip_local - c0, 0), hi - c0)
                stacks.append(LocalStack(self._blocks, self.x[c0:hi], self._rows[c0:hi], self._eps, ws=ws,
                                         skip=window))
            else:
                stacks.append(None)
        plan = (bounds, stacks, torch.cuda.Stream(self.send.device), torch.cuda.Stream(self.send.device))
        self._chunk_cache = (key, plan)
        return plan

    def forward_host(self, host_in: torch.Tensor, host_out: torch.Tensor | None = None,
                     chunks: int | None = None, *, shared_out: bool = False) -> None:
        """One end-to-end step from pinned host memory: this rank's input rows are
        copied in chunk by chunk on a copy stream while the block stack runs on the
        chunks already resident (every op is row-local).  Then either
          * (default) each chunk is gathered across ranks as soon as it is done and
            rank 0 (or the only rank) copies the gathered rows to ``host_out`` on a
            second copy stream, or
          * (``shared_out``: ``host_out`` is a node-shared pinned buffer of all
            [total, D] rows, see ``shared_host_output``) every rank copies its own
            finished rows into it over its own PCIe link -- no device gather; the
            output is complete when every rank has reached the end of this call.
        Everything is ordered on the current stream: when it reaches the end of
        this call's work, this rank's part of the output is in ``host_out``."""
        import torch.distributed as dist
        if host_in.shape != self.x.shape:
            raise ValueError(f"expected input shard {tuple(self.x.shape)}, got {tuple(host_in.shape)}")
        if shared_out and (host_out is None or host_out.shape[0] < self.total):
            raise ValueError("shared_out needs the node-shared [total, D] output buffer")
        # with every rank copying out its own rows, the copy-out share is one rank's
        bounds, stacks, h2d, d2h = self._chunking(chunks, schedule_world=1 if shared_out else self.world)
        comp = torch.cuda.current_stream(self.send.device)
        start = torch.cuda.Event()
        start.record(comp)
        h2d.wait_event(start)
        d2h.wait_event(start)
        arrived = []
        with torch.cuda.stream(h2d):
            for c0, c1 in bounds:
                hi = min(c1, self.rows_local)
                if hi > c0:
                    self.x[c0:hi].copy_(host_in[c0:hi], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(h2d)
                arrived.append(ev)
        multi = dist.is_initialized() and self.world > 1 and not shared_out
        for (c0, c1), stack, ev in zip(bounds, stacks, arrived):
            comp.wait_event(ev)
            if stack is not None:
                stack.run()
            rows = c1 - c0
            if multi:
                # chunk [c0, c1) of every rank, rank-major, in its own region of the
                # gather buffer: no region is reused within a call, so no gather
                # waits for an earlier chunk's copy out
                out = self.out[self.world * c0: self.world * c1]
                dist.all_gather_into_tensor(out, self.send[c0:c1], group=self.group)
            if host_out is None:
                continue
            done = torch.cuda.Event()
            done.record(comp)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                if not multi:
                    hi = min(c1, self.rows_local)
                    base = self.start if shared_out else 0
                    if hi > c0:
                        host_out[base + c0:base + hi].copy_(self.x[c0:hi], non_blocking=True)
                else:
                    for r in range(self.world):
                        g0, g1 = r * self.per + c0, min(self.total, r * self.per + c1)
                        if g1 > g0:
                            host_out[g0:g1].copy_(out[r * rows: r * rows + (g1 - g0)], non_blocking=True)
        comp.wait_stream(d2h)
        comp.wait_stream(h2d)
