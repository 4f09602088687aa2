"""KV-head sharding of the TT-KV read across ranks (one process per GPU).

The reference has no multi-GPU path; this is the build's. The read shards by KV head: after the
coefficient block every head's rows are independent. Rank g of N owns KV heads
[g*H/N, (g+1)*H/N) and either
* stores the storage-sharded format (`TTKLayout.shard`, `layout.shard_slots`): per token the
  coefficient block and its own heads' rows only, written by `ttkv_write_paged_shard` and read as
  a layout of H/N heads; or
* holds a replica of the full blobs and reads its heads through `head_lo/head_hi` of the read ABI.
Either way it writes its query heads [head_lo*G, head_hi*G) of each layer's output, which are
all-gathered over the process group and reassembled in head order, so every rank ends with the
whole output.

The write's projection needs every head's K (c = M @ pinv), so every rank projects the step's
tokens; with the sharded format it packs only its heads. Collectives go through
`torch.distributed` (NCCL on GPUs, gloo in the CPU tests), with the gathered tensor concatenated
along dim 0, the form both backends accept.
"""
from __future__ import annotations

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
