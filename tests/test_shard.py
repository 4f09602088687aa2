"""Head-sharded read across ranks, on the CPU with gloo (world size 2): each rank fills only its KV
heads' query heads of the output (here from the oracle restricted to those heads, standing in for
the read kernel's `head_lo/head_hi`), and `HeadShard.read` must leave the whole output on every
rank. Also: the head split itself, and a rank that fails before the collective ends the job with
an error instead of a hang."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vllm_ttkv.shard import HeadShard, head_range


def test_head_range_gives_every_head_to_exactly_one_rank():
    for world in (1, 2, 4, 8):
        got = [h for r in range(world) for h in range(*head_range(r, world, 8))]
        assert got == list(range(8))
    with pytest.raises(ValueError, match="do not divide"):
        head_range(0, 3, 8)
    with pytest.raises(ValueError):
        head_range(2, 2, 8)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _rank_reassembles(rank, world, port):
    from oracle import stores
    _init(rank, world, port)
    try:
        st = stores.make_store(11, [40, 23, 57], cfg="safe", r1=24)      # identical on every rank
        want = torch.from_numpy(stores.expected_decode(st))                 # [B, HQ, d]
        B, HQ, d = want.shape
        sh = HeadShard(8, HQ)
        assert (sh.head_lo, sh.head_hi) == head_range(rank, world, 8)

        def read_fn(lo, hi, out):                                          # this rank's heads only
            out[:, lo * sh.G:hi * sh.G] = want[:, lo * sh.G:hi * sh.G]

        out = torch.full((B, HQ, d), float("nan"))
        send, recv = sh.buffers(B, d, out.dtype, out.device)
        sh.read(read_fn, out, send, recv)
        assert torch.equal(out, want), f"rank {rank}: reassembled output differs"
    finally:
        dist.destroy_process_group()


def test_two_ranks_reassemble_the_whole_decode_output():
    mp.spawn(_rank_reassembles, args=(2, _free_port()), nprocs=2, join=True)


def _rank_fails_before_gather(rank, world, port):
    _init(rank, world, port, timeout_s=3)
    try:
        sh = HeadShard(8, 24)
        out = torch.zeros(2, 24, 128)
        send, recv = sh.buffers(2, 128, out.dtype, out.device)
        if rank == 1:
            raise RuntimeError("rank 1: refused its read")                 # never joins the gather
        sh.read(lambda lo, hi, o: None, out, send, recv)
    finally:
        dist.destroy_process_group()


def test_a_rank_that_fails_before_the_gather_ends_the_job_with_an_error():
    with pytest.raises(Exception):
        mp.spawn(_rank_fails_before_gather, args=(2, _free_port()), nprocs=2, join=True)
