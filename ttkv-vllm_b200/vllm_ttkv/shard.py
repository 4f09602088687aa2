"""KV-head sharding of the TT-KV read across ranks (one process per GPU).

The reference has no multi-GPU path; this is the build's. The read shards by KV head: after the
coefficient block every head's rows are independent. Rank g of N owns KV heads
[g*H/N, (g+1)*H/N) and either
* stores the storage-sharded format (`TTKLayout.shard`, `layout.shard_slots`): per token the
  coefficient block and its own heads' rows only, written by `ttkv_write_paged_shard` and read as
  a layout of H/N heads; or
* holds a replica of the full blobs and reads its heads through `head_lo/head_hi` of the read ABI.
Either way it writes its query heads [head_lo*G, head_hi*G) of each layer's output, and every rank
ends with the whole output: either `PeerGather`, where the decode's merge stores each row into
every rank's output over NVLink peer memory (no collective per layer), or `HeadShard.read`, an
all-gather over the process group reassembled in head order.

The write's projection needs every head's K (c = M @ pinv), so every rank projects the step's
tokens; with the sharded format it packs only its heads. Collectives go through
`torch.distributed` (NCCL on GPUs, gloo in the CPU tests), with the gathered tensor concatenated
along dim 0, the form both backends accept.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist


def request_range(rank: int, world: int, n_requests: int) -> tuple[int, int]:
    """Requests [lo, hi) a rank encodes when a prefill batch is split by request (the encode has
    no exchange: each request's fit and slots are its own). Contiguous shares in rank order, the
    first n_requests % world ranks taking one more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_requests < 0:
        raise ValueError("negative request count")
    base, extra = divmod(n_requests, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_bytes(local: torch.Tensor, group=None) -> torch.Tensor:
    """Every rank's uint8 tensor [n_r, C] concatenated in rank order on every rank (the byte
    comparison of a request-sharded encode). Shapes may differ across ranks in dim 0."""
    world = dist.get_world_size(group)
    n = torch.tensor([local.shape[0]], dtype=torch.int64, device=local.device)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n, group=group)
    counts = [int(c.item()) for c in counts]
    width = local.shape[1]
    pad = max(counts)
    buf = torch.zeros(pad, width, dtype=local.dtype, device=local.device)
    buf[:local.shape[0]] = local
    outs = [torch.zeros_like(buf) for _ in range(world)]
    dist.all_gather(outs, buf, group=group)
    return torch.cat([o[:c] for o, c in zip(outs, counts)])


def head_range(rank: int, world: int, H: int) -> tuple[int, int]:
    """KV heads [lo, hi) of `rank`: contiguous, equal shares in rank order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if H % world:
        raise ValueError(f"{world} ranks do not divide the {H} KV heads")
    n = H // world
    return rank * n, (rank + 1) * n


class HeadShard:
    """This rank's share of a head-sharded read and the all-gather that reassembles the output."""

    def __init__(self, H: int, HQ: int, world: int | None = None, rank: int | None = None, group=None):
        if HQ % H:
            raise ValueError(f"HQ={HQ} is not a multiple of H={H}")
        self.group = group
        self.world = dist.get_world_size(group) if world is None else int(world)
        self.rank = dist.get_rank(group) if rank is None else int(rank)
        self.H, self.HQ, self.G = H, HQ, HQ // H
        self.head_lo, self.head_hi = head_range(self.rank, self.world, H)
        self.q_lo, self.q_hi = self.head_lo * self.G, self.head_hi * self.G

    def buffers(self, B: int, d: int, dtype, device) -> tuple[torch.Tensor, torch.Tensor]:
        """(send [B, G*n, d], recv [world*B, G*n, d]) for one layer's output."""
        n = self.q_hi - self.q_lo
        return (torch.empty(B, n, d, dtype=dtype, device=device),
                torch.empty(self.world * B, n, d, dtype=dtype, device=device))

    def pack(self, out: torch.Tensor, send: torch.Tensor) -> None:
        """This rank's query heads of a layer output [B, HQ, d] into the send buffer."""
        send.copy_(out[:, self.q_lo:self.q_hi])

    def gather(self, send: torch.Tensor, recv: torch.Tensor) -> None:
        dist.all_gather_into_tensor(recv, send, group=self.group)

    def assemble(self, recv: torch.Tensor, out: torch.Tensor) -> None:
        """The gathered shares [world*B, G*n, d] into `out` [B, HQ, d], rank r's at its heads."""
        B, _, d = out.shape
        out.copy_(recv.view(self.world, B, -1, d).permute(1, 0, 2, 3).reshape(B, self.HQ, d))

    def read(self, read_fn, out: torch.Tensor, send: torch.Tensor, recv: torch.Tensor) -> torch.Tensor:
        """`read_fn(head_lo, head_hi, out)` writes this rank's query heads of `out`; afterwards `out`
        holds every head on every rank."""
        read_fn(self.head_lo, self.head_hi, out)
        self.pack(out, send)
        self.gather(send, recv)
        self.assemble(recv, out)
        return out


# ---------------------------------------------------------------------------- fused gather
def peers_struct(rank: int, outs, signals, epoch: int, ticket: int):
    """A `_lib.Peers` (ttkv_peers_t) from raw device addresses: every rank's output view and signal
    word as mapped in this process, and this rank's epoch and ticket words."""
    from vllm_ttkv import _lib
    world = len(outs)
    if world != len(signals) or not 1 <= world <= _lib.MAX_PEERS or not 0 <= rank < world:
        raise ValueError(f"a group of {world} outputs / {len(signals)} signals, rank {rank}")
    st = _lib.Peers()
    st.world, st.rank, st.epoch, st.ticket = world, rank, int(epoch), int(ticket)
    for i, (o, g) in enumerate(zip(outs, signals)):
        st.out[i], st.signal[i] = int(o), int(g)
    return st


class _DeviceArray:
    """Library-owned device memory as an int16 array, for a zero-copy `torch.as_tensor`."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<i2", "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class PeerGather:
    """The all-gather of a KV-head-sharded decode fused into its merge, over NVLink peer memory
    (`ttkv_decode_paged_gather` + `ttkv_peer_wait`): no NCCL call per layer.

    Every rank allocates, through CUDA IPC (plain peer mappings, no multicast object), one output
    buffer for all layers [L, B, HQ, d] (a 16- or 32-bit dtype) and one 8-byte signal word per
    layer, and keeps an epoch word and a ticket word per layer of its own. The handles are exchanged over the process group once and every rank
    maps the others'. Per layer and step, `ops.decode_paged(..., out=g.local_out(l),
    peers=g.peers(l))` stores this rank's query heads into every rank's buffer and counts its merge
    CTAs on every rank's signal word; `g.wait(l)` then waits (on the device, bounded) until this
    rank's buffer holds every head of the step: `g.out(l)` [B, HQ, d] (the step's requests in its
    first rows).

    Every rank must run the same layers and requests in the same order each step (the signal
    counts are cumulative; each rank's epoch word counts the arrivals its waits have taken).
    `lib` and `gather_object` stand in for the library and the collective in tests."""

    def __init__(self, shard: HeadShard, n_layers: int, B: int, d: int, dtype, device,
                 group=None, lib=None, gather_object=None):
        from vllm_ttkv import _lib
        self.shard, self.L, self.B, self.d = shard, int(n_layers), int(B), int(d)
        self.world, self.rank = shard.world, shard.rank
        self.device = torch.device(device)
        self._lib = lib if lib is not None else _lib.lib()
        self.esz = torch.tensor([], dtype=dtype).element_size()
        self.layer_bytes = self.B * shard.HQ * self.d * self.esz
        # every rank's merge CTAs (G x its KV heads x requests) arrive once per step
        self.per_request = self.world * shard.G * (shard.head_hi - shard.head_lo)
        self.arrivals = self.per_request * self.B
        self._own, self._opened = [], []
        hb = int(self._lib.ttkv_ipc_handle_bytes())

        def alloc(nbytes):
            ptr, h = C.c_void_p(), (C.c_char * hb)()
            _lib.check_with(self._lib, self._lib.ttkv_ipc_alloc(nbytes, C.byref(ptr), h))
            self._own.append(ptr.value)
            return ptr.value, bytes(h)

        base, h_out = alloc(self.L * self.layer_bytes)
        sig, h_sig = alloc(self.L * 8)
        handles = [None] * self.world
        if gather_object is None:
            dist.all_gather_object(handles, (h_out, h_sig), group=group)
        else:
            gather_object(handles, (h_out, h_sig))
        self.bases, self.signals = [], []
        for p, (ho, hs) in enumerate(handles):
            if p == self.rank:
                self.bases.append(base)
                self.signals.append(sig)
                continue
            pair = []
            for h in (ho, hs):
                ptr = C.c_void_p()
                _lib.check_with(self._lib, self._lib.ttkv_ipc_open(h, C.byref(ptr)))
                self._opened.append(ptr.value)
                pair.append(ptr.value)
            self.bases.append(pair[0])
            self.signals.append(pair[1])
        # per layer: the arrivals this rank's waits have taken, and its merge CTAs' ticket
        self.epoch = torch.zeros(self.L, dtype=torch.int64, device=self.device)
        self.ticket = torch.zeros(self.L, dtype=torch.int64, device=self.device)
        self.all_out = None
        if self.device.type == "cuda":
            raw = torch.as_tensor(_DeviceArray(base, (self.L, self.B, shard.HQ, self.d * self.esz // 2)),
                                  device=self.device)
            self.all_out = raw.view(dtype)                    # [L, B, HQ, d] of `dtype`
        q_off = shard.q_lo * self.d * self.esz
        self._peers = [peers_struct(self.rank, [b + l * self.layer_bytes + q_off for b in self.bases],
                                    [g + 8 * l for g in self.signals], self.epoch.data_ptr() + 8 * l,
                                    self.ticket.data_ptr() + 8 * l)
                       for l in range(self.L)]

    def out(self, l: int) -> torch.Tensor:
        """Layer l's whole output [B, HQ, d] on this rank (every head after `wait(l)`)."""
        return self.all_out[l]

    def local_out(self, l: int) -> torch.Tensor:
        """This rank's query heads of layer l's output: the `out` its decode writes."""
        return self.all_out[l][:, self.shard.q_lo:self.shard.q_hi]

    def peers(self, l: int):
        return self._peers[l]

    def wait(self, l: int, n_reqs: int | None = None, status=None) -> None:
        """Wait on the device for every rank's rows of layer l; `n_reqs`: the step's request count
        (every rank's), default the batch the buffers were sized for."""
        from vllm_ttkv import ops
        n = self.B if n_reqs is None else int(n_reqs)
        ops.peer_wait(self._peers[l], self.per_request * n, status)

    def close(self, group=None, barrier=None) -> None:
        """Unmap the peers' memory and free this rank's, once every rank is done with it (a group
        barrier first, or `barrier()` in tests)."""
        from vllm_ttkv import _lib
        if not self._own and not self._opened:
            return
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        (barrier or (lambda: dist.barrier(group)))()
        for ptr in self._opened:
            _lib.check_with(self._lib, self._lib.ttkv_ipc_close(ptr))
        self._opened = []
        (barrier or (lambda: dist.barrier(group)))()
        self.all_out = None
        for ptr in self._own:
            _lib.check_with(self._lib, self._lib.ttkv_ipc_free(ptr))
        self._own = []
