"""Per-step attention metadata for TT-KV: the batch description the attention impl reads
(vllm_ttkv/metadata.py:49-90 in the reference).

Every field is per step. vLLM hands one metadata object to every layer of a group, so anything the
impl derives from it once (the batch split, host copies of the block table) is cached on the object
under its `ttkv_serial`, and reused only while the serial matches.

`block_table[r, 0]` is also request r's identity: the key of its fitted decoder. `seq_lens` counts
each request's tokens INCLUDING the ones this step writes (the write runs before the read).
"""
from __future__ import annotations

import itertools
import os
from dataclasses import dataclass

import torch

try:                                   # vLLM's marker base classes when vLLM is installed
    from vllm.v1.attention.backend import AttentionMetadata as _MetadataBase
    from vllm.v1.attention.backend import AttentionMetadataBuilder as _BuilderBase
except Exception:                      # pragma: no cover - the impl itself does not need vLLM
    _MetadataBase = object
    _BuilderBase = object

_SERIAL = itertools.count(1)
# steps a request may go unnamed before the builder releases its decoders (0: never)
RELEASE_ENV = "VLLM_TTKV_RELEASE_AFTER"


def next_serial() -> int:
    return next(_SERIAL)


@dataclass
class TTKVAttentionMetadata(_MetadataBase):
    # [num_reqs] int32: exact token count of each request, including this step's tokens
    seq_lens: torch.Tensor | None = None
    # [num_tokens] int64: flat slot ids (block * block_size + offset) of this step's tokens
    slot_mapping: torch.Tensor | None = None
    # [num_reqs, max_blocks] int32: each request's blocks; column 0 is its decoder key
    block_table: torch.Tensor | None = None
    # [num_reqs + 1] int32: cumulative query lengths (decodes first)
    query_start_loc: torch.Tensor | None = None
    query_start_loc_cpu: torch.Tensor | None = None
    # an upper bound of seq_lens on the host (never used as a row count)
    seq_lens_cpu_upper_bound: torch.Tensor | None = None
    positions: torch.Tensor | None = None
    num_actual_tokens: int = 0
    max_query_len: int = 0
    max_seq_len: int = 0
    # set by build(); 0 = not built here, and the impl then recomputes its plan per layer
    ttkv_serial: int = 0


def build(common, positions=None) -> TTKVAttentionMetadata:
    """Copy a step's metadata off vLLM's `CommonAttentionMetadata` (or any object with its field
    names) and stamp the next serial."""
    bt = getattr(common, "block_table_tensor", None)
    if bt is None:
        bt = getattr(common, "block_table", None)
    return TTKVAttentionMetadata(
        seq_lens=common.seq_lens,
        slot_mapping=common.slot_mapping,
        block_table=bt,
        query_start_loc=common.query_start_loc,
        query_start_loc_cpu=getattr(common, "query_start_loc_cpu", None),
        seq_lens_cpu_upper_bound=getattr(common, "seq_lens_cpu", None),
        positions=positions,
        num_actual_tokens=int(getattr(common, "num_actual_tokens", 0)),
        max_query_len=int(getattr(common, "max_query_len", 0)),
        max_seq_len=int(getattr(common, "max_seq_len", 0)),
        ttkv_serial=next_serial())


class TTKVAttentionMetadataBuilder(_BuilderBase):
    """vLLM's per-step builder: decodes are reordered to the front of the batch
    (`reorder_batch_threshold = 1`), which the impl verifies; speculative decoding is refused."""

    reorder_batch_threshold: int = 1

    def __init__(self, kv_cache_spec=None, layer_names=None, vllm_config=None, device=None):
        if _BuilderBase is not object:
            super().__init__(kv_cache_spec, layer_names, vllm_config, device)
        if vllm_config is not None and getattr(vllm_config, "speculative_config", None) is not None:
            raise NotImplementedError(
                "TT-KV does not support speculative decoding: drafted tokens are not stored keys.")
        from vllm_ttkv import rope_store
        self._reaper = rope_store.AbsenceReaper(int(os.environ.get(RELEASE_ENV, "0") or 0))

    def build(self, common_prefix_len, common_attn_metadata, fast_build: bool = False):
        md = build(common_attn_metadata)
        if self._reaper.after > 0 and md.block_table is not None and md.seq_lens is not None:
            n = int(md.seq_lens.shape[0])           # one readback per step, only when enabled
            self._reaper.step(md.block_table[:n, 0].tolist())
        return md

    @staticmethod
    def release_finished(keys) -> None:
        """Return the decoders of finished requests, named by their keys (the first block id of
        each request's block-table row, read before the engine frees the blocks): every layer's
        pool row goes back to the free list and the device key map forgets the key."""
        from vllm_ttkv import rope_store
        for k in keys:
            rope_store.release_request(int(k))
