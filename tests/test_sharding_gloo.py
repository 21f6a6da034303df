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
