"""Multi-rank host logic on CPU: two gloo ranks run the sharded DCN path the way
`bench.py --gpus N` does (each rank regenerates its own block of images from
(seed, global image index) and computes it alone, no collective on the data
path), and the result equals the single-rank run of all images.  The kernels
are replaced by the CPU oracle here; the GPU kernels are covered by the -m gpu
tests.  Also checks the max-over-ranks timing reduction."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

SEED = 77
N_IMAGES = 5  # not a multiple of the world size: blocks of 3 and 2
CFG = dict(C=16, H=9, W=11, Cout=24, dtype="float32", big=0.05)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dcn_block(b0, n, oracle, bench):
    """Output of images [b0, b0 + n) generated and computed by one rank."""
    if n == 0:
        return np.zeros((0, CFG["Cout"], CFG["H"], CFG["W"]), np.float32)
    s = bench.dcn_sets(dict(CFG, B=n), 1, SEED, b0, "cpu")[0]
    return oracle.dcn_forward(s["x"], s["off"], s["mask"], s["w"], None, 1, 1, 1,
                              nthreads=1)


def _worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        from bevk.sharding import shard_range
        from oracle import oracle
        b0, b1 = shard_range(N_IMAGES, rank, world)
        mine = _dcn_block(b0, b1 - b0, oracle, bench)
        # outside any timed region: collect the blocks on every rank
        blocks = [None] * world
        dist.all_gather_object(blocks, (b0, mine))
        got = np.concatenate([blk for _, blk in sorted(blocks, key=lambda t: t[0])])
        want = _dcn_block(0, N_IMAGES, oracle, bench)
        assert got.shape == want.shape
        assert np.array_equal(got, want), "sharded result differs from the single-rank run"
        # timing reduction: every rank sees the slowest rank's time
        slowest = bench._max_over_ranks(10.0 + rank, dist)
        assert slowest == 10.0 + world - 1
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _gather_worker(rank, world, port, total):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        from bevk.sharding import shard_range
        b0, b1 = shard_range(total, rank, world)
        # rank r holds rows [b0, b1) of a table whose row i is (i, 10 i)
        mine = torch.tensor([[float(i), 10.0 * i] for i in range(b0, b1)],
                            dtype=torch.float64).reshape(-1, 2)
        table = bench.gather_rows(mine, total, rank, world, dist)
        want = torch.tensor([[float(i), 10.0 * i] for i in range(total)], dtype=torch.float64)
        assert torch.equal(table, want)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total", [(2, 48), (3, 7), (4, 3)])
def test_chain_checksum_gather(world, total):
    """The 5-chain's checksum table: each rank's block of rows (unequal blocks,
    empty ones) reaches every rank in image order."""
    mp.spawn(_gather_worker, args=(world, _free_port(), total), nprocs=world, join=True)


def test_two_gloo_ranks_shard_dcn_like_one_rank():
    port = _free_port()
    mp.spawn(_worker, args=(2, port), nprocs=2, join=True)


def test_shard_blocks_match_bench_image_seeds():
    """A rank's block regenerates exactly the same cameras as the world-1 run."""
    import bench
    whole = bench.dcn_sets(dict(CFG, B=N_IMAGES), 1, SEED, 0, "cpu")[0]
    part = bench.dcn_sets(dict(CFG, B=2), 1, SEED, 3, "cpu")[0]
    for k in ("x", "off", "mask"):
        assert torch.equal(part[k], whole[k][3:5])
    assert torch.equal(part["w"], whole["w"])


def test_chain_blocks_match_world_one_images():
    """A rank's block of the 5-chain regenerates exactly the same images (MSDA
    camera slices and DCN images) as the world-1 run, and shares its weight."""
    import bench
    whole_m, whole_d = bench.chain_inputs(0, 3, SEED, "cpu")
    part_m, part_d = bench.chain_inputs(1, 2, SEED, "cpu")
    for k in ("value", "loc", "attn"):
        assert torch.equal(part_m[k], whole_m[k][1:3])
    for k in ("shapes", "lsi"):
        assert torch.equal(part_m[k], whole_m[k])
    for k in ("x", "off", "mask"):
        assert torch.equal(part_d[k], whole_d[k][1:3])
    assert torch.equal(part_d["w"], whole_d["w"])
