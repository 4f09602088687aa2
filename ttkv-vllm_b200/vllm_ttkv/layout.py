"""What one cache slot holds: the per-token TT-KV byte layout of a layer.

Same surface as the reference's `vllm_ttkv/layout.py` (TTKLayout, align_up, packed_row_bytes,
layout_for_config, pack/unpack_{k,v}_slots), because the slot format is the drop-in boundary:
a cache written by either implementation must read back identically through the other.

One token's blob is [K slot][V slot]:
    K slot = [r1 int8 coefficients][fp16 coefficient ruler][H x (d/8 bitmap, packed codes, fp16)]
    V slot = [H x (d/8 bitmap, packed codes, fp16 ruler)]
each padded to `align` bytes (vllm_ttkv/layout.py:56-157). Residual and V rows are in
(head, token) = h*n + i order in the codec containers and token-major in the slots.
"""
from __future__ import annotations

import ctypes
import dataclasses
import math
from dataclasses import dataclass

import torch

# The three allocations of the codec (codec/ttkv_codec.py:272-298). Format parameters: they decide
# slot widths, so the numbers are the reference's.
CONFIGS = {
    "safe": dict(tols=0.20, qbits=8, res_frac=0.633, res_bits=3, k_lanes=81, vbits=3),
    "tight": dict(tols=0.20, qbits=8, res_frac=0.25, res_bits=3, k_lanes=45, vbits=3),
    "campaign4x": dict(tols=0.20, qbits=8, res_frac=0.50, res_bits=4, k_lanes=64, vbits=4),
}
# deprecated names of the same allocations (codec/ttkv_codec.py:246-256)
CONFIG_ALIASES = {"loose_late": "campaign4x", "core8": "tight", "balanced": "safe"}


def config(name: str) -> dict:
    name = CONFIG_ALIASES.get(name, name)
    if name not in CONFIGS:
        raise KeyError(f"{name!r} is not a config and is not a deprecated alias")
    return CONFIGS[name]


def align_up(n: int, a: int) -> int:
    return n if a <= 1 else ((n + a - 1) // a) * a


def packed_row_bytes(k: int, bits: int) -> int:
    """Each row of codes is padded to whole bytes."""
    return math.ceil(k * bits / 8)


@dataclass(frozen=True)
class TTKLayout:
    """Byte layout of one layer's TT-KV cache; every size is PER TOKEN."""

    H: int
    d: int
    r1: int
    qbits: int
    res_k: int
    res_bits: int
    v_lanes: int
    v_bits: int
    align: int = 16

    def __post_init__(self):
        if self.d % 8:
            raise ValueError(
                f"head dim {self.d} is not a multiple of 8; the lane bitmap is d/8 bytes per row")
        if self.res_k > self.d:
            raise ValueError(f"res_k={self.res_k} exceeds d={self.d}")
        if self.v_lanes > self.d:
            raise ValueError(
                f"v_lanes={self.v_lanes} exceeds d={self.d}: `k_lanes` is an absolute lane count "
                f"and has to be re-derived for a narrower head")

    @property
    def coeff_bytes(self) -> int:
        if (self.r1 * self.qbits) % 8:
            raise ValueError(f"r1={self.r1} at qbits={self.qbits} is not a whole number of bytes")
        return self.r1 * self.qbits // 8

    @property
    def k_row_bytes(self) -> int:
        return self.d // 8 + packed_row_bytes(self.res_k, self.res_bits) + 2

    @property
    def v_row_bytes(self) -> int:
        return self.d // 8 + packed_row_bytes(self.v_lanes, self.v_bits) + 2

    @property
    def coeff_scale_bytes(self) -> int:
        return 2

    @property
    def v_offset(self) -> int:
        return self.k_slot_bytes

    @property
    def k_slot_bytes(self) -> int:
        return align_up(self.coeff_bytes + self.coeff_scale_bytes + self.H * self.k_row_bytes,
                        self.align)

    @property
    def v_slot_bytes(self) -> int:
        return align_up(self.H * self.v_row_bytes, self.align)

    def dense_bytes_per_token(self) -> int:
        return 2 * self.H * self.d * 2

    def compressed_bytes_per_token(self) -> int:
        return self.k_slot_bytes + self.v_slot_bytes

    def ratio(self) -> float:
        return self.dense_bytes_per_token() / self.compressed_bytes_per_token()

    def shard(self, h_lo: int, h_hi: int) -> "TTKLayout":
        """The layout of a storage-sharded cache that holds only KV heads [h_lo, h_hi): the same
        widths with H = h_hi - h_lo, i.e. the coefficient block and its ruler, then the held heads'
        K rows (padded to `align`), then their V rows (padded). No counterpart in the reference,
        which has no multi-GPU path; the reassembled shards are the reference's slot bytes
        (`shard_slots` / `unshard_slots`)."""
        if not 0 <= h_lo < h_hi <= self.H:
            raise ValueError(f"heads [{h_lo}, {h_hi}) outside the layout's {self.H}")
        if (h_lo, h_hi) == (0, self.H):
            return self
        return dataclasses.replace(self, H=h_hi - h_lo)

    def abi(self):
        """The `ttkv_layout_t` of this layout, validated by the library."""
        from vllm_ttkv import _lib
        cached = getattr(self, "_abi", None)
        if cached is not None:
            return cached
        st = _lib.Layout()
        _lib.check(_lib.lib().ttkv_layout_init(
            ctypes.byref(st), self.H, self.d, self.r1, self.qbits, self.res_k, self.res_bits,
            self.v_lanes, self.v_bits, self.align))
        assert st.blob_bytes == self.compressed_bytes_per_token()
        object.__setattr__(self, "_abi", st)
        return st


def layout_for_config(cfg, r1: int, H: int = 8, d: int = 128) -> TTKLayout:
    """A layout from a config (dict or name) plus the layer's rank budget
    (vllm_ttkv/layout.py:264-275)."""
    if isinstance(cfg, str):
        cfg = config(cfg)
    return TTKLayout(H=H, d=d, r1=r1, qbits=cfg["qbits"],
                     res_k=max(int(d * cfg["res_frac"]), 1), res_bits=cfg["res_bits"],
                     v_lanes=cfg["k_lanes"], v_bits=cfg["vbits"])


# ---------------------------------------------------------------- the storage-sharded format
def shard_slots(rows: torch.Tensor, lay: TTKLayout, h_lo: int, h_hi: int) -> torch.Tensor:
    """The shard of full blobs `rows` [n, >= blob_bytes] uint8 that holds KV heads [h_lo, h_hi):
    [n, lay.shard(h_lo, h_hi).blob_bytes], padding zero."""
    sl = lay.shard(h_lo, h_hi)
    head = lay.coeff_bytes + 2
    out = torch.zeros(rows.shape[0], sl.compressed_bytes_per_token(), dtype=torch.uint8, device=rows.device)
    out[:, :head] = rows[:, :head]
    nk, nv = (h_hi - h_lo) * lay.k_row_bytes, (h_hi - h_lo) * lay.v_row_bytes
    out[:, head:head + nk] = rows[:, head + h_lo * lay.k_row_bytes:head + h_hi * lay.k_row_bytes]
    out[:, sl.v_offset:sl.v_offset + nv] = rows[:, lay.v_offset + h_lo * lay.v_row_bytes:
                                                lay.v_offset + h_hi * lay.v_row_bytes]
    return out


def unshard_slots(shards, lay: TTKLayout, ranges) -> torch.Tensor:
    """Full blobs [n, lay.blob_bytes] from shards [n, >= shard blob] holding the KV head ranges
    `ranges` (together every head once): the coefficient block of the first shard, each head's
    rows from the shard holding it, padding zero."""
    covered = sorted(h for lo, hi in ranges for h in range(lo, hi))
    if covered != list(range(lay.H)):
        raise ValueError(f"the head ranges {list(ranges)} do not cover the {lay.H} heads exactly once")
    head = lay.coeff_bytes + 2
    n = shards[0].shape[0]
    out = torch.zeros(n, lay.compressed_bytes_per_token(), dtype=torch.uint8, device=shards[0].device)
    out[:, :head] = shards[0][:, :head]
    for rows, (lo, hi) in zip(shards, ranges):
        sl = lay.shard(lo, hi)
        nk, nv = (hi - lo) * lay.k_row_bytes, (hi - lo) * lay.v_row_bytes
        out[:, head + lo * lay.k_row_bytes:head + hi * lay.k_row_bytes] = rows[:, head:head + nk]
        out[:, lay.v_offset + lo * lay.v_row_bytes:lay.v_offset + hi * lay.v_row_bytes] = \
            rows[:, sl.v_offset:sl.v_offset + nv]
    return out


# ---------------------------------------------------------------- the codec's row container
class PackedRows:
    """A [rows, d] block as bitmap + k packed codes + one fp16 ruler per row (the container of
    codec/ttkv_packed_cache.py:186-271, fields only)."""

    def __init__(self, rows: int, d: int, k: int, bits: int, bitmap=None, packed=None, scale=None):
        self.rows, self.d, self.k, self.bits = rows, d, k, bits
        self.bitmap, self.packed, self.scale = bitmap, packed, scale


def _u8(t: torch.Tensor, n: int) -> torch.Tensor:
    return t.contiguous().view(torch.uint8).reshape(n, -1)


def pack_k_slots(lay: TTKLayout, coeff_q, coeff_scale, resid: PackedRows) -> torch.Tensor:
    """[n, k_slot_bytes] uint8 from int8 coefficients [n, r1], fp16 rulers [n] and a residual
    container over H*n (head, token) rows."""
    n = coeff_q.shape[0]
    if resid.rows != lay.H * n:
        raise ValueError(f"residual holds {resid.rows} rows, expected H*n = {lay.H * n}")
    out = torch.zeros(n, lay.k_slot_bytes, dtype=torch.uint8, device=coeff_q.device)
    out[:, :lay.coeff_bytes] = _u8(coeff_q.to(torch.int8), n)
    out[:, lay.coeff_bytes:lay.coeff_bytes + 2] = _u8(coeff_scale.to(torch.float16), n)
    _put_rows(out, lay.coeff_bytes + 2, lay.H, n, resid)
    return out


def pack_v_slots(lay: TTKLayout, rows: PackedRows) -> torch.Tensor:
    n = rows.rows // lay.H
    if rows.rows % lay.H:
        raise ValueError(f"V store holds {rows.rows} rows, not a multiple of H={lay.H}")
    out = torch.zeros(n, lay.v_slot_bytes, dtype=torch.uint8, device=rows.bitmap.device)
    _put_rows(out, 0, lay.H, n, rows)
    return out


def _put_rows(out, off, H, n, pr: PackedRows):
    b, p = pr.bitmap.shape[1], pr.packed.shape[1]
    step = b + p + 2
    for h in range(H):
        s = slice(h * n, (h + 1) * n)
        base = off + h * step
        out[:, base:base + b] = pr.bitmap[s]
        out[:, base + b:base + b + p] = pr.packed[s]
        out[:, base + b + p:base + step] = _u8(pr.scale[s].to(torch.float16), n)


def _get_rows(slots, off, H, d, k, bits) -> PackedRows:
    n = slots.shape[0]
    b, p = d // 8, packed_row_bytes(k, bits)
    step = b + p + 2
    rows = [slots[:, off + h * step: off + (h + 1) * step] for h in range(H)]
    blk = torch.cat(rows, 0) if rows else slots.new_zeros(0, step)
    return PackedRows(H * n, d, k, bits, blk[:, :b].contiguous(), blk[:, b:b + p].contiguous(),
                      blk[:, b + p:].contiguous().view(torch.float16).reshape(H * n))


def unpack_k_slots(lay: TTKLayout, slots: torch.Tensor):
    """Inverse of pack_k_slots: (coeff_q int8 [n, r1], coeff_scale fp16 [n], PackedRows)."""
    n = slots.shape[0]
    cq = slots[:, :lay.coeff_bytes].contiguous().view(torch.int8)
    cs = slots[:, lay.coeff_bytes:lay.coeff_bytes + 2].contiguous().view(torch.float16).reshape(n)
    return cq, cs, _get_rows(slots, lay.coeff_bytes + 2, lay.H, lay.d, lay.res_k, lay.res_bits)


def unpack_v_slots(lay: TTKLayout, slots: torch.Tensor) -> PackedRows:
    return _get_rows(slots, 0, lay.H, lay.d, lay.v_lanes, lay.v_bits)
