"""Request-sharded encode across ranks, on the CPU with gloo (world size 2): each rank encodes only
its share of the requests (the oracle's fit + slot packing stands in for the device encoder), with
no exchange; the gathered slot bytes must equal a single process encoding every request, byte for
byte. Also the request split itself."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vllm_ttkv.shard import gather_bytes, request_range


def test_request_range_gives_every_request_to_exactly_one_rank():
    for world in (1, 2, 3, 4, 8):
        for n in (0, 1, 5, 8, 13):
            got = [r for k in range(world) for r in range(*request_range(k, world, n))]
            assert got == list(range(n)), (world, n)
            sizes = [len(range(*request_range(k, world, n))) for k in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        request_range(2, 2, 4)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _encode(r):
    """Request r's packed slots (the oracle's encoder on its own seeded keys)."""
    from oracle import ttkv_oracle as O
    from vllm_ttkv import synthetic as S
    g = O.geometry_for_config("tight", 16)
    K, V = S.synth_kv(500 + r, 40)
    f = O.fit_into_budget(K, g, "tight")
    return O.build_slots(g, f["coeff_q"], f["coeff_scale"], f["R"], V)


def _rank_encodes_its_share(rank, world, port, n_req):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        lo, hi = request_range(rank, world, n_req)
        mine = [_encode(r) for r in range(lo, hi)]
        local = torch.from_numpy(np.concatenate(mine) if mine else np.zeros((0, 640), np.uint8))
        allb = gather_bytes(local).numpy()
        want = np.concatenate([_encode(r) for r in range(n_req)])
        assert np.array_equal(allb, want), f"rank {rank}: gathered slot bytes differ"
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_req", [2, 3])
def test_two_ranks_encode_their_requests_and_the_bytes_reassemble(n_req):
    mp.spawn(_rank_encodes_its_share, args=(2, _free_port(), n_req), nprocs=2, join=True)
