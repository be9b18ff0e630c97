"""Multi-rank plumbing of bench.py on CPU: world_size 2 (and 3) with gloo.

The data path has no collective; ranks only agree on their token / sequence
shards and take the max of their timings. These tests run the same functions
the benchmark uses, in real spawned ranks."""

import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench

        t0, tn = bench.shard(262144, rank, world)
        s0, sn = bench.shard(64, rank, world)
        m = bench.max_over_ranks(float(10 * (rank + 1)), world)
        bench.barrier(world)
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
        rc = bench.reference_arm(bench.parse_args(["--impl", "reference", "--steps", "1", "--warmup", "0"]),
                                 rank, world) if rank != 0 else 0
        out.put((rank, t0, tn, s0, sn, m, rc))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ranks_shard_tokens_and_sequences_and_agree_on_max(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    starts = [r[1] for r in res]
    sizes = [r[2] for r in res]
    assert starts[0] == 0 and sum(sizes) == 262144
    assert all(starts[i] + sizes[i] == starts[i + 1] for i in range(world - 1))
    assert max(sizes) - min(sizes) <= 1
    seq = [r[4] for r in res]
    assert sum(seq) == 64 and max(seq) - min(seq) <= 1
    assert all(r[5] == 10.0 * world for r in res)  # every rank sees the max over ranks
    assert all(r[6] == 0 for r in res)  # the reference arm: non-zero ranks exit 0 without work
