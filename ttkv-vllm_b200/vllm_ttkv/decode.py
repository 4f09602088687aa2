"""Read-side conventions and guards (the reference's `vllm_ttkv/decode.py` surface).

The hot path does not gather, split or expand anything here: `ops.decode_paged` and
`ops.prefill_cont_paged` read the paged cache in place. What remains are the conventions the
kernels share with vLLM -- the cos/sin table layout, the byte view of a page, the slot-id
arithmetic -- the host-side refusals, and the first-chunk prefill, which is plain causal SDPA over
the model's own post-RoPE q/k/v exactly as in the reference (decode.py:363-389).
"""
from __future__ import annotations

import torch

from vllm_ttkv.layout import TTKLayout

__all__ = ["cos_sin_from_cache", "byte_rows", "block_slots", "check_row_host", "repeat_kv",
           "check_layout_matches_decoder", "check_row_counts", "attend_prefill", "gather_slots",
           "split_blob"]


def cos_sin_from_cache(cos_sin_cache: torch.Tensor, positions: torch.Tensor, head_dim: int,
                       rotary_dim: int | None = None, max_position: int | None = None):
    """`(cos, sin)` [n, head_dim] fp32 in the duplicated (j, j + d/2) frame from vLLM's
    `cat(cos, sin)` table (decode.py:54-122). The kernels read the table directly; this is the
    convention spelled out for callers and tests."""
    rot = cos_sin_cache.shape[-1] if rotary_dim is None else rotary_dim
    if rot != head_dim:
        raise NotImplementedError(
            f"rotary_dim={rot} != head_dim={head_dim} (partial rotary): the kernels pair (j, j+d/2) "
            f"across the whole row; refusing rather than rotating the wrong lanes")
    rows = cos_sin_cache.shape[0]
    if max_position is not None and max_position >= rows:
        raise IndexError(f"position {max_position} is past the model's cos_sin_cache, which holds "
                         f"{rows} entries")
    row = cos_sin_cache[positions.to(torch.long)].to(torch.float32)
    c, s = row[:, :rot // 2], row[:, rot // 2:]
    return torch.cat([c, c], -1).contiguous(), torch.cat([s, s], -1).contiguous()


def byte_rows(page: torch.Tensor, slot_bytes: int, what: str = "the KV cache") -> torch.Tensor:
    """`[slots, W]` uint8 rows of a paged cache tensor, W >= slot_bytes (decode.py:125-157): the
    page is allocated in the model dtype with its width counted in elements."""
    try:
        u8 = page if page.dtype == torch.uint8 else page.view(torch.uint8)
    except RuntimeError as e:
        raise RuntimeError(f"{what} of shape {tuple(page.shape)} and dtype {page.dtype} cannot be "
                           f"viewed as bytes ({e})") from e
    if u8.shape[-1] < slot_bytes:
        raise ValueError(f"{what} has a slot width of {u8.shape[-1]} bytes but this layout needs "
                         f"{slot_bytes}; a write would land in the next token's row")
    return u8.reshape(-1, u8.shape[-1])


def block_slots(block_row: torch.Tensor, seq_len: int, block_size: int) -> torch.Tensor:
    """Flat slot ids of a request's first seq_len tokens: block*block_size + offset."""
    if seq_len < 0:
        raise ValueError(f"seq_len={seq_len} is negative")
    pos = torch.arange(seq_len, device=block_row.device)
    return block_row[pos // block_size].to(torch.long) * block_size + pos % block_size


def check_row_host(row, seq_len: int, block_size: int, n_slots: int | None = None) -> None:
    """The three refusals of a block-table row already on the host (decode.py:200-234)."""
    if seq_len < 0:
        raise ValueError(f"seq_len={seq_len} is negative")
    if seq_len == 0:
        return
    n_blocks = -(-seq_len // block_size)
    if n_blocks > len(row):
        raise IndexError(f"seq_len={seq_len} needs {n_blocks} blocks of {block_size} but the block "
                         f"table row holds {len(row)}")
    used = row[:n_blocks]
    if min(used) < 0:
        raise IndexError(f"the block table row holds {min(used)} inside its used prefix")
    if n_slots is not None and max(used) * block_size >= n_slots:
        raise IndexError(f"block {max(used)} is outside the cache, which holds "
                         f"{n_slots // block_size} blocks of {block_size}")


def repeat_kv(x: torch.Tensor, G: int) -> torch.Tensor:
    if G == 1:
        return x
    T, Hkv, d = x.shape
    return x[:, :, None, :].expand(T, Hkv, G, d).reshape(T, Hkv * G, d)


def check_layout_matches_decoder(lay: TTKLayout, decoder_f: torch.Tensor) -> None:
    got = int(decoder_f.shape[0])
    if lay.r1 != got:
        raise ValueError(f"the layout says r1={lay.r1} but the fitted decoder has r1={got} rows; "
                         f"the slot width is derived from r1")


def check_row_counts(k_rows: int, v_rows: int, cos_rows: int, seq_len: int) -> None:
    if not (k_rows == v_rows == cos_rows == seq_len):
        raise RuntimeError(f"row counts disagree with the request: K={k_rows}, V={v_rows}, "
                           f"angles={cos_rows}, seq_len={seq_len}")


def gather_slots(cache_layer: torch.Tensor, slots: torch.Tensor, slot_bytes: int | None = None):
    """`[n, slot_bytes]` copies of the named slots (for inspection and tests; the kernels never
    gather)."""
    c = cache_layer[:, 0] if cache_layer.dim() == 4 else cache_layer
    want = c.shape[-1] if slot_bytes is None else slot_bytes
    flat = byte_rows(c, want)
    return flat[slots, :want].contiguous()


def split_blob(lay: TTKLayout, blob: torch.Tensor):
    k = lay.k_slot_bytes
    if blob.shape[-1] != k + lay.v_slot_bytes:
        raise ValueError(f"a token's blob is {blob.shape[-1]} bytes but the layout asks for "
                         f"{k} + {lay.v_slot_bytes}")
    return blob[:, :k].contiguous(), blob[:, k:].contiguous()


def attend_prefill(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   scale: float) -> torch.Tensor:
    """First-chunk prefill: causal SDPA over the model's post-RoPE q/k/v, [T, HQ, d] out."""
    G = query.shape[1] // key.shape[1]
    if query.shape[1] != key.shape[1] * G:
        raise ValueError(f"num_heads={query.shape[1]} is not a multiple of num_kv_heads={key.shape[1]}")
    q = query.transpose(0, 1).unsqueeze(0)
    k = repeat_kv(key, G).transpose(0, 1).unsqueeze(0)
    v = repeat_kv(value, G).transpose(0, 1).unsqueeze(0)
    out = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale)
    return out.squeeze(0).transpose(0, 1).contiguous()
