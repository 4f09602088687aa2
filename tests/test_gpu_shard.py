"""The storage-sharded decode step of bench.py's multi-GPU path, one rank at a time on one GPU: a
rank that stores only its KV heads' rows writes the step's tokens (bytes that reassemble to the
full write's) and reads its query heads (outputs equal to the full read's on those heads)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _workload():
    import bench
    return bench.Workload(2, 300, [32, 110], "safe", torch.device("cuda", 0), torch.bfloat16, seed=3)


def _copy(wl):
    """The same stores, decoders and inputs (one fit), with caches and outputs of its own."""
    import copy
    c = copy.copy(wl)
    c.caches = [x.clone() for x in wl.caches]
    c.out = [x.clone() for x in wl.out]
    c.images = list(wl.images)
    c.read_layouts = list(wl.read_layouts)
    c.read_dec = list(wl.read_dec)
    return c


@pytest.mark.parametrize("world", [2, 8])
def test_a_rank_storing_its_heads_writes_and_reads_like_the_full_store(world):
    from vllm_ttkv import ops
    from vllm_ttkv.layout import unshard_slots
    from vllm_ttkv.shard import head_range
    full = _workload()
    ranks = []
    for r in range(world):
        wl = _copy(full)
        lo, hi = head_range(r, world, wl.H)
        wl.shard(lo, hi)
        ranks.append((wl, (lo, hi)))
    ops.reset_status()
    for l in range(full.L):
        full.layer_step(l)
    for wl, _ in ranks:
        for l in range(wl.L):
            wl.layer_step(l)
    torch.cuda.synchronize()
    ops.check_status()
    G = full.HQ // full.H
    for l in range(full.L):
        got = unshard_slots([wl.caches[l] for wl, _ in ranks], full.layouts[l], [hr for _, hr in ranks])
        assert torch.equal(got, full.caches[l][:, :full.layouts[l].compressed_bytes_per_token()]), l
        for wl, (lo, hi) in ranks:
            a = wl.out[l][:, lo * G:hi * G].float().cpu().numpy()
            b = full.out[l][:, lo * G:hi * G].float().cpu().numpy()
            np.testing.assert_allclose(a, b, rtol=1e-2, atol=1e-3, err_msg=f"{l} {lo}")  # bf16 outputs
