"""Token sharding on two GPUs (NCCL), run as two spawned processes.

Skipped unless the box shows at least two GPUs.  Rank r owns the contiguous
token block shard_bounds(M, 2, r); the gathered output of the device-resident
forward, of the chunk-pipelined end-to-end forward (pinned host in, rank 0
host out) and of the same with a node-shared pinned output that every rank
fills with its own rows must equal one GPU running every row, bit for bit.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

D, FFN = 512, 1024


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, result_path, chunks=3):
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "comfyui-h3-speedkit_b200"), str(root / "tests")]
    import torch.distributed as dist
    from h3_speedkit import synthetic
    from h3_speedkit.stack import LocalStack, ShardedStack, shard_bounds
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        blocks = [synthetic.cfg5_block(i, D, FFN).to(dev) for i in range(2)]
        x_all = synthetic.cfg5_tokens(m, D)
        start, stop = shard_bounds(m, world, rank)
        rows = torch.zeros((stop - start,), dtype=torch.int32, device=dev)
        stack = ShardedStack(blocks, rows, m, D, dev)
        stack.load(x_all[start:stop].to(dev))
        gathered = stack.forward().cpu()
        host_in = x_all[start:stop].contiguous().pin_memory()
        host_out = torch.empty((m, D), dtype=torch.bfloat16).pin_memory() if rank == 0 else None
        for _ in range(2):
            stack.forward_host(host_in, host_out, chunks=chunks)
        torch.cuda.synchronize()
        # node-shared pinned output: every rank writes its own rows, no gather
        from h3_speedkit.stack import shared_host_output
        shared = shared_host_output(m, D)
        assert shared is not None
        for _ in range(2):
            stack.forward_host(host_in, shared, chunks=chunks, shared_out=True)
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            ref = x_all.to(dev)
            LocalStack(blocks, ref, torch.zeros((m,), dtype=torch.int32, device=dev)).run()
            torch.cuda.synchronize()
            ok = (torch.equal(gathered, ref.cpu()) and torch.equal(host_out, ref.cpu())
                  and torch.equal(shared, ref.cpu()))
            Path(result_path).write_text("ok" if ok else "mismatch")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m,chunks", [(1001, 3), (20011, None)])
def test_two_gpu_token_sharding_matches_one_gpu(tmp_path, m, chunks):
    """(20011, None): 10006 rows per rank take the ramped chunk schedule, with a
    ragged last shard and a chunk that is not a multiple of 128 rows."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    result = tmp_path / "result.txt"
    mp.spawn(_worker, args=(2, _free_port(), m, str(result), chunks), nprocs=2, join=True)
    assert result.read_text() == "ok"
