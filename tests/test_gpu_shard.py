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


def test_the_gathered_decode_leaves_every_head_on_every_rank():
    """`ttkv_decode_paged_gather` for two ranks emulated on one GPU: each rank's merge stores its
    query heads into both ranks' outputs and counts on both signal words; after both ranks' reads
    (one stream, so every wait below finds its arrivals already counted) `ttkv_peer_wait` passes
    and each output holds every head, equal to the full read. Two steps: the second waits for the
    second epoch's arrivals."""
    from vllm_ttkv import ops
    from vllm_ttkv.shard import head_range, peers_struct
    world = 2
    full = _workload()
    ranks = []
    for r in range(world):
        wl = _copy(full)
        wl.shard(*head_range(r, world, wl.H))
        ranks.append(wl)
    B, HQ, d, L, G = full.B, full.HQ, 128, full.L, full.HQ // full.H
    outs = [torch.full((L, B, HQ, d), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(world)]
    sigs = [torch.zeros(L, dtype=torch.int64, device="cuda") for _ in range(world)]
    epochs = [torch.zeros(L, dtype=torch.int64, device="cuda") for _ in range(world)]
    tickets = [torch.zeros(L, dtype=torch.int64, device="cuda") for _ in range(world)]
    arrivals = world * G * (full.H // world) * B
    ops.reset_status()
    for step in range(2):
        for l in range(L):
            full.layer_step(l)
            structs = []
            for r, wl in enumerate(ranks):
                lo, hi = head_range(r, world, wl.H)
                st = peers_struct(r, [o[l].data_ptr() + lo * G * d * 2 for o in outs],
                                  [g.data_ptr() + 8 * l for g in sigs], epochs[r].data_ptr() + 8 * l,
                                  tickets[r].data_ptr() + 8 * l)
                structs.append(st)
                wl.write(l)
                ops.decode_paged(wl.read_layouts[l], wl.caches[l], wl.bs, wl.block_table, wl.seq_lens,
                                 wl.read_dec[l], wl.dec_index, wl.table, wl.q[l][:, lo * G:hi * G],
                                 wl.scale, outs[r][l][:, lo * G:hi * G], wl.max_seq,
                                 images=wl.images[l], peers=st)
            for st in structs:
                ops.peer_wait(st, arrivals)
        torch.cuda.synchronize()
        ops.check_status()
        for r in range(world):
            assert int(sigs[r][0].item()) == (step + 1) * arrivals
            assert int(epochs[r][0].item()) == (step + 1) * arrivals
            assert int(tickets[r].abs().sum().item()) == 0              # every launch's last CTA reset it
            for l in range(L):
                np.testing.assert_allclose(outs[r][l].float().cpu().numpy(), full.out[l].float().cpu().numpy(),
                                           rtol=1e-2, atol=1e-3, err_msg=f"rank {r} layer {l} step {step}")


def test_a_peer_wait_with_no_arrivals_runs_out_and_reports():
    """A signal word nobody counts on: the bounded wait gives up after about two seconds, sets
    TTKV_STATUS_TIMEOUT and still counts the step's arrivals as waited for; the device stays
    usable."""
    import time

    from vllm_ttkv import _lib, ops
    from vllm_ttkv.shard import peers_struct
    out = torch.zeros(1, 8, 128, dtype=torch.bfloat16, device="cuda")
    sig = torch.zeros(1, dtype=torch.int64, device="cuda")
    ep = torch.zeros(1, dtype=torch.int64, device="cuda")
    tk = torch.zeros(1, dtype=torch.int64, device="cuda")
    st = peers_struct(0, [out.data_ptr()], [sig.data_ptr()], ep.data_ptr(), tk.data_ptr())
    ops.reset_status()
    t0 = time.perf_counter()
    ops.peer_wait(st, 3)
    torch.cuda.synchronize()
    assert 0.5 < time.perf_counter() - t0 < 30
    assert int(ops.status_word().item()) == 6          # TTKV_STATUS_TIMEOUT
    assert int(ep.item()) == 3
    ops.reset_status()
    sig.fill_(3 + 5)                                   # the next step of 5 arrivals: the wait passes
    ops.peer_wait(st, 5)
    torch.cuda.synchronize()
    ops.check_status()
    assert int(ep.item()) == 8
    with pytest.raises(_lib.TTKVError):
        ops.peer_wait(peers_struct(0, [out.data_ptr()], [sig.data_ptr()], 0, tk.data_ptr()), 3)   # no epoch word
