"""Token sharding of the block stack across ranks, on CPU ranks over gloo.

Every op of the path is row-local, so contiguous token shards computed
independently and gathered must equal the unsharded result bit for bit.  Each
rank runs the CPU restatement of the block chain on its shard (the GPU ranks
run the CUDA kernels through the same shard bookkeeping and gather).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from h3_speedkit import synthetic
from h3_speedkit.stack import gather_shards, shard_bounds

D, FFN, BLOCKS = 512, 1024, 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(total):
    from oracle.chain import NpBlock
    blocks = [NpBlock.from_torch(synthetic.cfg5_block(i, D, FFN, tables=2)) for i in range(BLOCKS)]
    x = synthetic.cfg5_tokens(total, D).view(torch.int16).numpy().view(np.uint16)
    rows = (np.arange(total) % 2).astype(np.int32)
    return blocks, x, rows


def _rank_main(rank, world, port, total, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import chain
        blocks, x, rows = _inputs(total)
        start, stop = shard_bounds(total, world, rank)
        per = -(-total // world)
        send = torch.zeros((per, D), dtype=torch.int16)
        if stop > start:
            out = chain.stack(x[start:stop].copy(), blocks, rows[start:stop].copy(), threads=1)
            send[: stop - start] = torch.from_numpy(out.view(np.int16))
        # gloo has no 16-bit types: move the BF16 bit patterns as int32 pairs
        gathered = torch.empty((per * world, D // 2), dtype=torch.int32)
        full = gather_shards(send.view(torch.int32), gathered, total)
        if rank == 0:
            np.save(result_path, full.numpy().view(np.int16))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total", [(2, 48), (2, 37)])
def test_sharded_stack_equals_unsharded(tmp_path, world, total):
    from oracle import chain
    result = tmp_path / "gathered.npy"
    mp.start_processes(_rank_main, args=(world, _free_port(), total, str(result)), nprocs=world, join=True,
                       start_method="spawn")
    gathered = np.load(result).view(np.uint16)
    blocks, x, rows = _inputs(total)
    reference = chain.stack(x.copy(), blocks, rows, threads=1)
    assert gathered.shape == reference.shape
    assert np.array_equal(gathered, reference)


def test_shard_bounds_cover_every_token_once():
    for total in (1, 7, 98304, 98305):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and a <= b
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def test_chunk_schedule_covers_the_shard_with_small_end_chunks():
    """The end-to-end pipeline's chunks cover [0, per) once, in order; the first
    and last chunks are the smallest; the tail never shrinks faster than the
    copy-out share allows (up to the 128-row rounding), and every chunk but one
    is a multiple of 128 rows."""
    from h3_speedkit.stack import chunk_schedule
    for per in (1, 1001, 7000, 8192, 12288, 16128, 24576, 30000, 49152, 98304, 98305):
        for world in (1, 2, 4, 8):
            bounds = chunk_schedule(per, world)
            assert bounds[0][0] == 0 and bounds[-1][1] == per
            for (a, b), (c, d) in zip(bounds, bounds[1:]):
                assert b == c and a < b
            sizes = [b - a for a, b in bounds]
            if per < 8 * 1024:
                assert len(sizes) <= 4
                continue
            small = max(1024, -(-(per // 16) // 128) * 128)
            assert sizes[0] == small and sizes[-1] == small
            assert sum(s % 128 != 0 for s in sizes) <= 1
            down = min(0.8, max(0.25, 0.1 * world))
            tail = sizes[sizes.index(max(sizes)):]
            for prev, nxt in zip(tail, tail[1:]):
                assert nxt >= down * prev - 128


def test_oracle_row_window_is_the_block_on_the_window():
    """chain.block(skip=s): rows < s copied through, rows >= s the block on them alone."""
    from oracle import chain
    m, skip = 40, 16
    b = chain.NpBlock.from_torch(synthetic.cfg5_block(0, 256, 512, tables=2))
    x = np.ascontiguousarray(synthetic.cfg5_tokens(m, 256).view(torch.int16).numpy().view(np.uint16))
    rows = (np.arange(m) % 2).astype(np.int32)
    full = chain.block(x, b, rows, threads=1)
    win = chain.block(x, b, rows, threads=1, skip=skip)
    assert np.array_equal(win[:skip], x[:skip])
    assert np.array_equal(win[skip:], full[skip:])


def _shared_worker(rank, world, port, directory, result_dir):
    import os as _os
    _os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from h3_speedkit.stack import shared_host_output
        out = shared_host_output(16, 32, group=None, directory=directory)
        # on a host without a CUDA device the mapping cannot be page-locked: every
        # rank agrees on None, and the file is gone
        with open(f"{result_dir}/r{rank}", "w") as fh:
            fh.write("none" if out is None else "tensor")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_shared_host_output_agrees_across_ranks_without_a_gpu(tmp_path):
    """shared_host_output on CPU ranks: every rank takes the same collective steps,
    all return None when page-locking is impossible, and the shared file is removed."""
    if torch.cuda.is_available():
        pytest.skip("checks the fallback of a host without a CUDA device")
    shm = tmp_path / "shm"
    shm.mkdir()
    mp.spawn(_shared_worker, args=(2, _free_port(), str(shm), str(tmp_path)), nprocs=2, join=True)
    assert (tmp_path / "r0").read_text() == "none" and (tmp_path / "r1").read_text() == "none"
    assert list(shm.iterdir()) == []


def test_shared_host_output_without_room_returns_none(tmp_path, monkeypatch):
    import os
    from h3_speedkit.stack import shared_host_output

    class Full:
        f_bavail, f_frsize = 1, 4096
    monkeypatch.setattr(os, "statvfs", lambda path: Full())
    assert shared_host_output(1024, 1024, directory=str(tmp_path)) is None
    assert list(tmp_path.iterdir()) == []
