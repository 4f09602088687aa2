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


class _FakeIpcLib:
    """Stands in for the library's CUDA IPC calls on a CPU: an allocation is a fresh fake address
    per rank, its handle names it, and opening a handle maps it at an address of this rank's."""

    def __init__(self, rank):
        self.rank, self.next, self.log = rank, 0x10000000 * (rank + 1), []

    def ttkv_ipc_handle_bytes(self):
        return 64

    def ttkv_ipc_alloc(self, nbytes, ptr, handle):
        ptr._obj.value = self.next
        tag = f"{self.rank}:{self.next:x}:{nbytes}".encode()
        handle[:len(tag)] = tag
        self.log.append(("alloc", self.next, nbytes))
        self.next += 0x1000000
        return 0

    def ttkv_ipc_open(self, handle, ptr):
        rank, addr, _ = bytes(handle).rstrip(b"\0").decode().split(":")
        ptr._obj.value = 0x900000000 + int(rank) * 0x10000000 + int(addr, 16) % 0x10000000
        self.log.append(("open", int(rank), int(addr, 16)))
        return 0

    def ttkv_ipc_close(self, ptr):
        self.log.append(("close", ptr))
        return 0

    def ttkv_ipc_free(self, ptr):
        self.log.append(("free", ptr))
        return 0

    def ttkv_last_error(self):
        return b""


def _rank_peer_tables(rank, world, port):
    from vllm_ttkv.shard import PeerGather
    _init(rank, world, port)
    try:
        B, HQ, d, L = 3, 24, 128, 4
        sh = HeadShard(8, HQ)
        fake = _FakeIpcLib(rank)
        g = PeerGather(sh, L, B, d, torch.bfloat16, "cpu", lib=fake)
        layer = B * HQ * d * 2
        assert g.arrivals == world * sh.G * (8 // world) * B == sh.G * 8 * B
        own = [a for op, a, n in fake.log if op == "alloc"]
        assert [n for op, a, n in fake.log if op == "alloc"] == [L * layer, L * 8]
        opened = [(r, a) for op, r, a in fake.log if op == "open"]
        assert sorted({r for r, _ in opened}) == [p for p in range(world) if p != rank]
        for l in range(L):
            st = g.peers(l)
            assert (st.world, st.rank) == (world, rank)
            assert st.epoch == g.epoch.data_ptr() + 8 * l
            assert st.ticket == g.ticket.data_ptr() + 8 * l
            for p in range(world):
                base = g.bases[p]
                assert st.out[p] == base + l * layer + sh.q_lo * d * 2       # this rank's head view
                assert st.signal[p] == g.signals[p] + 8 * l
            assert st.out[rank] == own[0] + l * layer + sh.q_lo * d * 2
        g.close(barrier=dist.barrier)
        assert [op for op, *_ in fake.log[-3:]] == ["close", "free", "free"] or world == 1
    finally:
        dist.destroy_process_group()


def test_peer_gather_maps_every_ranks_output_and_signal_words():
    """The fused gather's host side on two gloo ranks: one IPC allocation for the outputs of all
    layers and one for the signal words, the handles exchanged, every other rank's memory mapped,
    and per layer a ttkv_peers_t whose out[p] is rank p's output at this rank's head offset."""
    mp.spawn(_rank_peer_tables, args=(2, _free_port()), nprocs=2, join=True)


def test_peers_struct_refuses_mismatched_or_oversized_groups():
    from vllm_ttkv import _lib
    from vllm_ttkv.shard import peers_struct
    st = peers_struct(1, [0x1000, 0x2000], [0x3000, 0x4000], 0x5000, 0x6000)
    assert (st.world, st.rank, st.epoch, st.ticket) == (2, 1, 0x5000, 0x6000)
    assert list(st.out)[:2] == [0x1000, 0x2000] and list(st.signal)[:2] == [0x3000, 0x4000]
    with pytest.raises(ValueError):
        peers_struct(0, [1, 2], [3], 4, 5)                          # one signal for two outputs
    with pytest.raises(ValueError):
        peers_struct(2, [1, 2], [3, 4], 5, 6)                       # rank outside the group
    n = _lib.MAX_PEERS + 1
    with pytest.raises(ValueError):
        peers_struct(0, list(range(1, n + 1)), list(range(1, n + 1)), 1, 1)
