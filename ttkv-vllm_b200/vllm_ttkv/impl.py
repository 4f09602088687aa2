"""`TTKVAttentionImpl`: the vLLM attention impl over the TT-KV packed store (the drop-in for
vllm_ttkv/impl.py:325-498 of the reference).

`forward(layer, query, key, value, kv_cache, attn_metadata, output)` is called once per layer per
step. It WRITES this step's tokens into the store, then READS attention for every request, and
fills `output` in place (vLLM discards a return value).

Per layer, the work is a handful of launches whatever the batch holds:

* write: requests that already have a fitted decoder (decodes, continuation chunks) are projected
  onto it and packed in ONE `ttkv_write_paged` launch pair (device decoder pool, one pool row per
  request); a request on its first chunk gets its TT-SVD fit (`encode.fit_into_budget`), is
  written, and its decoder is registered for the steps after (vllm_ttkv/impl.py:543-658).
* decode: ONE `ttkv_decode_paged` launch for all requests with one query token (the reference
  loops over requests, impl.py:468-493).
* prefill: a first chunk attends over its own post-RoPE q/k/v by SDPA (decode.py:363-389); all
  continuation chunks (seq_len > q_len) read the store in ONE `ttkv_prefill_cont_paged` launch
  (impl.py:725-778).

The step's layer-independent facts (batch split, request keys, bounds of the slot mapping) are read
back once per step and cached on the metadata under its serial (impl.py:82-214). Device-side
refusals (a block id outside the cache, a decoder row outside the pool) land in `ops.status_word`;
with VLLM_TTKV_CHECK=1 every layer reads it back and raises.

A pure-decode step (every query length 1, seen in the host copy of query_start_loc) can instead be
planned on the device (`DevicePlan`): each request's pool row comes from the device key map, the
read's bound is the RoPE table's length, and nothing is read back, so the forward can be captured
in a CUDA graph and replayed for later steps of the same request count. That is the plan while a
graph is being captured, and always with VLLM_TTKV_DEVICE_PLAN=1. The host-side refusals of the
other plan (PAD_SLOT_ID or out-of-range slots, a request without a decoder) then become device
refusals in the status word, read by `ops.check_status()`, except that a PAD_SLOT_ID slot is
skipped: an engine padding a decode batch to a captured size gives its padding tokens that slot
(and seq_len 0, which the read skips). The reference's backend cannot be captured at all
(vllm_ttkv/metadata.py:95-101).
"""
from __future__ import annotations

import os

import torch

from vllm_ttkv import decode as dc
from vllm_ttkv import encode, ops
from vllm_ttkv.layout import TTKLayout
from vllm_ttkv.patch import take_raw_k
from vllm_ttkv.rope_store import (decoder_for_request, ensure_store, key_rows, layout_for_layer,
                                  pool_for_layer, register_decoder, request_key_host, request_slot,
                                  rows_for_keys)

try:                                   # vLLM's base class when vLLM is installed
    from vllm.v1.attention.backend import AttentionImpl as _ImplBase
except Exception:                      # pragma: no cover
    _ImplBase = object

try:
    from vllm.v1.attention.backend import AttentionType as _AttentionType
except Exception:                      # pragma: no cover
    _AttentionType = None

_CHECK = os.environ.get("VLLM_TTKV_CHECK", "") not in ("", "0")
_DEVICE_PLAN = os.environ.get("VLLM_TTKV_DEVICE_PLAN", "") not in ("", "0")
_SIDE_STREAMS: dict = {}        # device -> the stream first chunks' attention runs on
_PLAN_ATTR = "_ttkv_plan"


def validate_slot_ids(slot_mapping: torch.Tensor, n_tokens: int, n_slots: int) -> None:
    """The write's refusals on the whole step's slot ids (one readback per step,
    impl.py:217-238): PAD_SLOT_ID (< 0) and slots outside the cache."""
    if n_tokens <= 0:
        return
    ids = slot_mapping[:n_tokens]
    lo, hi = (int(x) for x in torch.stack([ids.min(), ids.max()]).tolist())
    if lo < 0:
        raise RuntimeError(
            f"slot_mapping contains {lo}, i.e. vLLM's PAD_SLOT_ID: a padded token has no cache slot, "
            f"so its key cannot be stored, and the read covers exactly seq_len rows. Refusing.")
    if hi >= n_slots:
        raise IndexError(f"slot {hi} is outside the cache, which holds {n_slots} slots")


class StepPlan:
    """Everything about a step that does not depend on the layer, read back and checked once."""

    __slots__ = ("serial", "qsl", "seq_lens", "n_reqs", "n_dec", "prefills", "keys", "block_size",
                 "n_slots", "_dec_rows", "_cont", "_frozen")

    def __init__(self, md, block_size: int, n_slots: int, serial: int):
        if md.query_start_loc is None or md.seq_lens is None or md.block_table is None:
            raise RuntimeError(
                "the attention metadata is missing query_start_loc / seq_lens / block_table, so the "
                "batch cannot be split or addressed")
        if md.slot_mapping is None:
            raise RuntimeError("the metadata carries no slot_mapping, so there is nowhere to write")
        self.serial = serial
        qsl_src = md.query_start_loc_cpu if md.query_start_loc_cpu is not None else md.query_start_loc
        self.qsl = [int(x) for x in qsl_src.tolist()]
        # exact row counts come from the device tensor: the CPU copy is only an upper bound
        self.seq_lens = [int(x) for x in md.seq_lens.tolist()]
        if len(self.qsl) != len(self.seq_lens) + 1:
            raise RuntimeError(
                f"query_start_loc has {len(self.qsl)} entries but seq_lens has {len(self.seq_lens)}")
        self.n_reqs = len(self.seq_lens)
        if md.block_table.shape[0] < self.n_reqs:
            raise RuntimeError(
                f"the block table has {md.block_table.shape[0]} rows for {self.n_reqs} requests")
        q_len = [self.qsl[i + 1] - self.qsl[i] for i in range(self.n_reqs)]
        decodes = [r for r, ql in enumerate(q_len) if ql == 1]
        self.n_dec = len(decodes)
        if decodes != list(range(self.n_dec)):
            raise RuntimeError(
                f"decode requests are not contiguous at the front of the batch (decode rows "
                f"{decodes}, query lengths {q_len}); vLLM's reorder puts them there")
        self.prefills = [r for r in range(self.n_reqs) if q_len[r] > 1]
        self.block_size, self.n_slots = block_size, n_slots
        # a request's identity is its first block (the key of its decoder)
        self.keys = [int(x) for x in md.block_table[:self.n_reqs, 0].tolist()] if self.n_reqs else []
        validate_slot_ids(md.slot_mapping, self.qsl[-1], n_slots)
        self._dec_rows = None
        self._cont = None
        self._frozen = {}

    def frozen_write(self, frozen: tuple, device):
        """(token rows, pool row per token) of the write for the frozen requests `frozen` (request,
        pool row) pairs; the same for every layer of the step, so built once. Token rows are a
        (start, end) range when the requests are contiguous, else an index tensor."""
        got = self._frozen.get(frozen)
        if got is None:
            reqs = [r for r, _ in frozen]
            counts = torch.tensor([self.qsl[r + 1] - self.qsl[r] for r in reqs])
            rows = torch.repeat_interleave(torch.tensor([p for _, p in frozen], dtype=torch.int32),
                                           counts).to(device)
            if reqs == list(range(reqs[0], reqs[-1] + 1)):
                tok = (self.qsl[reqs[0]], self.qsl[reqs[-1] + 1])
            else:
                tok = torch.cat([torch.arange(self.qsl[r], self.qsl[r + 1]) for r in reqs]).to(device)
            got = (tok, rows)
            self._frozen[frozen] = got
        return got

    def dec_rows(self, device) -> torch.Tensor:
        """Pool rows of the decode requests (the same row in every layer)."""
        if self._dec_rows is None:
            rows = [request_slot(self.keys[r]) for r in range(self.n_dec)]
            missing = [self.keys[r] for r, s in enumerate(rows) if s is None]
            if missing:
                raise RuntimeError(
                    f"no fitted TT-KV decoder for request(s) {missing}: a decoder is created by the "
                    f"write of a request's first chunk, so these requests never had one")
            self._dec_rows = torch.tensor(rows, dtype=torch.int32, device=device)
        return self._dec_rows


def decode_only(md) -> int:
    """The request count of a pure-decode step (every query length 1), from the HOST copy of
    query_start_loc; 0 when the step is anything else or there is no host copy."""
    qc = getattr(md, "query_start_loc_cpu", None)
    if qc is None or qc.is_cuda or qc.dim() != 1 or qc.numel() < 2:
        return 0
    n = qc.numel() - 1
    return n if torch.equal(qc, torch.arange(n + 1, dtype=qc.dtype)) else 0


class DevicePlan:
    """A pure-decode step planned without a readback: request r is token r, its pool row is
    looked up on the device from its key (`block_table[r, 0]`), and the read is bounded by the
    RoPE table rather than by the batch's longest request."""

    __slots__ = ("serial", "n", "block_size", "n_slots", "captured", "_rows")

    def __init__(self, md, n: int, block_size: int, n_slots: int, serial: int, captured: bool):
        if md.seq_lens is None or md.block_table is None or md.slot_mapping is None:
            raise RuntimeError(
                "the attention metadata is missing seq_lens / block_table / slot_mapping, so the "
                "batch cannot be addressed")
        if md.seq_lens.shape[0] < n or md.block_table.shape[0] < n or md.slot_mapping.shape[0] < n:
            raise RuntimeError(
                f"a decode step of {n} requests needs {n} seq_lens, block-table rows and slots "
                f"(got {md.seq_lens.shape[0]}, {md.block_table.shape[0]}, {md.slot_mapping.shape[0]})")
        if md.block_table.shape[1] < 1:
            raise ValueError("the block table has no columns, so no request has an identity to key "
                             "a decoder by")
        self.serial, self.n, self.block_size, self.n_slots = serial, n, block_size, n_slots
        # made under a capture: its row lookup is a node of the graph, redone at every replay
        self.captured = captured
        self._rows = None

    def rows(self, md, device) -> torch.Tensor:
        """Pool row of each request (-1: no decoder, refused on the device), made once per step."""
        if self._rows is None:
            key_rows(device, self.n_slots // self.block_size)
            self._rows = rows_for_keys(md.block_table[:self.n, 0])
        return self._rows


def plan_for(md, block_size: int, n_slots: int, device_plan: bool = False, capturing: bool = False):
    """The step's plan, cached on the metadata under its serial. A device plan made outside a
    capture is not reused inside one (its row lookup must be captured too), nor the other way."""
    n_dec = decode_only(md) if device_plan else 0
    serial = int(getattr(md, "ttkv_serial", 0) or 0)
    plan = getattr(md, _PLAN_ATTR, None) if serial else None
    if plan is not None and plan.serial == serial:
        if isinstance(plan, DevicePlan) and n_dec and plan.captured == capturing:
            return plan
        if isinstance(plan, StepPlan) and not n_dec:
            return plan
    plan = (DevicePlan(md, n_dec, block_size, n_slots, serial, capturing) if n_dec
            else StepPlan(md, block_size, n_slots, serial))
    if serial:
        setattr(md, _PLAN_ATTR, plan)
    return plan


class TTKVAttentionImpl(_ImplBase):
    def __init__(self, num_heads: int, head_size: int, scale: float, num_kv_heads: int | None = None,
                 alibi_slopes=None, sliding_window=None, kv_cache_dtype: str = "auto",
                 logits_soft_cap=None, attn_type=None, kv_sharing_target_layer_name=None, **kwargs):
        # each of these would change the scores or the keys attended, silently (impl.py:326-349)
        if alibi_slopes is not None:
            raise NotImplementedError("TT-KV does not support ALiBi: the read has no bias term")
        if logits_soft_cap is not None:
            raise NotImplementedError("TT-KV does not support logits_soft_cap")
        if sliding_window is not None:
            raise NotImplementedError(
                "TT-KV does not support a sliding window: the read attends over the whole store")
        if kv_sharing_target_layer_name is not None:
            raise NotImplementedError(
                "TT-KV does not support KV sharing: another layer's store has a different decoder")
        if _AttentionType is not None and attn_type is not None and attn_type != _AttentionType.DECODER:
            raise NotImplementedError(f"TT-KV only supports decoder attention, got {attn_type!r}")
        self.num_heads = num_heads
        self.head_size = head_size
        self.num_kv_heads = num_kv_heads or num_heads
        self.scale = float(scale)
        self.kv_cache_dtype = kv_cache_dtype
        if num_heads % self.num_kv_heads:
            raise ValueError(f"num_heads={num_heads} is not a multiple of num_kv_heads={self.num_kv_heads}")

    # ------------------------------------------------------------------ the entry point
    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output=None,
                output_scale=None, output_block_scale=None):
        """`query` [N, HQ, d] post-RoPE; `key`/`value` [N, H*d or H, d] (key post-RoPE, used for
        a first chunk only); `kv_cache` the layer's page [blocks, 1, block_size, C]. Writes
        `output` [N, HQ, d] in place."""
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("TT-KV does not support fused output quantization")
        if attn_metadata is None:
            if output is None:
                raise ValueError("attn_metadata and output are both None; there is nothing to write")
            return output.fill_(0)
        n_tokens = query.shape[0]
        if output is None:
            output = torch.empty(n_tokens, self.num_heads, self.head_size, dtype=query.dtype,
                                 device=query.device)
        lay = self._layout(layer)
        page = self._cache_tensor(kv_cache)
        block_size = self._block_size(page)
        cache = dc.byte_rows(page, lay.compressed_bytes_per_token())
        capturing = ops.capturing()
        if query.is_cuda and not capturing:          # any eager step readies a later capture
            key_rows(query.device, cache.shape[0] // block_size)
        plan = plan_for(attn_metadata, block_size, cache.shape[0], _DEVICE_PLAN or capturing, capturing)
        if isinstance(plan, DevicePlan):
            if plan.n > n_tokens:
                raise RuntimeError(f"metadata describes {plan.n} query tokens but the query holds {n_tokens}")
            self._decode_step(layer, lay, cache, plan, attn_metadata, query, value, output, capturing)
            if _CHECK and not capturing:
                ops.check_status(query.device)
            return output
        N = plan.qsl[-1]
        actual = getattr(attn_metadata, "num_actual_tokens", None)
        if actual and int(actual) != N:
            raise RuntimeError(
                f"query_start_loc says {N} query tokens but num_actual_tokens says {actual}")
        if N > n_tokens:
            raise RuntimeError(f"metadata describes {N} query tokens but the query holds {n_tokens}")
        if N == 0:
            return output
        name = getattr(layer, "layer_name", None)
        # first chunks attend over their own q/k/v, which the write does not change: their SDPA
        # goes out first, on a side stream, and runs under the fits (whose rank choice reads back
        # to the host) and the writes; the step's stream waits for it before returning
        side = self._first_chunks_aside(plan, query, key, value, output)
        table = self._write(layer, name, lay, cache, value, plan, attn_metadata, query.device)
        if plan.n_dec:
            self._decode(name, lay, cache, plan, attn_metadata, table, query, output)
        if plan.prefills:
            self._prefill(name, lay, cache, plan, attn_metadata, table, query, key, value, output,
                          skip_first=side is not None)
        if side is not None:
            torch.cuda.current_stream(query.device).wait_stream(side)
        if _CHECK:
            ops.check_status(query.device)
        return output

    def _first_chunks_aside(self, plan, query, key, value, output):
        """Launch the first chunks' attention on a side stream (CUDA only); None when there are
        none, or off CUDA, or under a capture (the side stream is not part of it)."""
        if not query.is_cuda or ops.capturing():
            return None
        firsts = [r for r in plan.prefills if plan.seq_lens[r] == plan.qsl[r + 1] - plan.qsl[r]]
        if not firsts:
            return None
        cur = torch.cuda.current_stream(query.device)
        side = _SIDE_STREAMS.get(query.device)
        if side is None:                            # one per device, made once
            side = _SIDE_STREAMS[query.device] = torch.cuda.Stream(device=query.device)
        side.wait_stream(cur)                       # q/k/v are the step stream's
        with torch.cuda.stream(side):
            self._attend_first_chunks(firsts, plan, query, key, value, output)
        for t in (query, key, value, output):       # used on the side stream
            if t is not None:
                t.record_stream(side)
        return side

    def _attend_first_chunks(self, firsts, plan, query, key, value, output):
        for r in firsts:
            s, e = plan.qsl[r], plan.qsl[r + 1]
            k = encode.as_kv_heads(key, self.num_kv_heads, self.head_size, "key")[s:e].float()
            v = encode.as_kv_heads(value, self.num_kv_heads, self.head_size, "value")[s:e].float()
            out = dc.attend_prefill(query[s:e].float(), k, v, self.scale)
            output[s:e] = out.to(output.dtype)

    # ------------------------------------------------------------------ a device-planned decode step
    def _decode_step(self, layer, lay, cache, plan, md, query, value, output, capturing):
        """Write token r of every request r and read every request, with no host readback: the
        frozen write and the decode, each request's pool row from the device key map."""
        name = getattr(layer, "layer_name", None)
        stash = take_raw_k(name)
        if value is None:
            raise RuntimeError(f"layer {name!r} got no value tensor, so V cannot be stored")
        if lay.H != self.num_kv_heads:
            raise RuntimeError(
                f"the layout was built for H={lay.H} KV heads but this layer has {self.num_kv_heads}")
        n, dev = plan.n, query.device
        K = encode.as_kv_heads(stash["raw_k"], self.num_kv_heads, self.head_size, "the captured raw key")[:n]
        V = encode.as_kv_heads(value, self.num_kv_heads, self.head_size, "value")[:n]
        table = self._device_table(self._cos_sin_cache(layer, stash), query)
        ensure_store(name, table, self.num_heads, self.num_kv_heads, self.head_size, lay)
        pool = pool_for_layer(name, lay, dev)
        rows = plan.rows(md, dev)
        if capturing:                       # the graph holds these addresses from now on
            pool.pin()
            ops.pin(key_rows(dev), rows)
        # a batch padded to a captured size carries PAD_SLOT_ID for its padding tokens: skipped
        encode.write_frozen(cache, md.slot_mapping[:n], K, V, rows, pool.decoders, pool.pinvT, lay,
                            skip_pad=True)
        # the read's bound: the RoPE table (any position the model can reach) under a capture, so
        # the replays of other lengths stay within it; else the step's own max_seq_len
        bound = int(table.shape[0])
        if not capturing and 0 < int(getattr(md, "max_seq_len", 0) or 0) <= bound:
            bound = int(md.max_seq_len)
        ops.decode_paged(lay, cache, plan.block_size, md.block_table[:n], md.seq_lens[:n],
                         pool.decoders, rows, table, query[:n], self.scale, output[:n], bound,
                         images=pool.images)

    # ------------------------------------------------------------------ the write
    def _write(self, layer, name, lay, cache, value, plan, md, device):
        """Encode this step's raw K and V into the store; returns the layer's RoPE table."""
        stash = take_raw_k(name)
        if value is None:
            raise RuntimeError(f"layer {name!r} got no value tensor, so V cannot be stored")
        if lay.H != self.num_kv_heads:
            raise RuntimeError(
                f"the layout was built for H={lay.H} KV heads but this layer has {self.num_kv_heads}")
        N = plan.qsl[-1]
        K = encode.as_kv_heads(stash["raw_k"], self.num_kv_heads, self.head_size, "the captured raw key")[:N]
        V = encode.as_kv_heads(value, self.num_kv_heads, self.head_size, "value")[:N]
        table = self._cos_sin_cache(layer, stash)
        ensure_store(name, table, self.num_heads, self.num_kv_heads, self.head_size, lay)
        slots = md.slot_mapping[:N]
        frozen = []                      # (request, pool row)
        for r in range(plan.n_reqs):
            s, e = plan.qsl[r], plan.qsl[r + 1]
            if e <= s:
                continue
            k = plan.keys[r]
            # a first chunk (all of the request's tokens are in this step) is always fitted: a
            # decoder already under its key belongs to a finished request whose first block the
            # engine has since handed to this one, and projecting onto it would store this
            # request's keys in another request's basis. The refit overwrites it in place (same
            # pool row). The reference reuses the stale decoder here (impl.py:614).
            first = plan.seq_lens[r] == e - s
            if not first and decoder_for_request(name, k) is not None:
                frozen.append((r, request_slot(k)))
                continue
            if not first:
                raise RuntimeError(
                    f"request {k} has seq_len={plan.seq_lens[r]} but {e - s} tokens in this step and "
                    f"no fitted decoder: a continuation whose first chunk was never written")
            fk = encode.fit_into_budget(K[s:e].permute(1, 0, 2).contiguous(), lay, encode.active_config())
            encode.write_fitted(cache, slots[s:e].contiguous(), fk, K[s:e], V[s:e], lay)
            register_decoder(name, k, fk.decoder, lay=lay)
        if frozen:
            pool = pool_for_layer(name, lay, device)
            tok, rows = plan.frozen_write(tuple(frozen), device)
            if isinstance(tok, tuple):              # the usual case: every request frozen, in order
                s, e = tok
                encode.write_frozen(cache, slots[s:e], K[s:e], V[s:e], rows, pool.decoders,
                                    pool.pinvT, lay)
            else:
                encode.write_frozen(cache, slots.index_select(0, tok), K.index_select(0, tok),
                                    V.index_select(0, tok), rows, pool.decoders, pool.pinvT, lay)
        return table

    # ------------------------------------------------------------------ the reads
    def _decode(self, name, lay, cache, plan, md, table, query, output):
        """All decode requests (rows 0..n_dec-1) in one launch; rows read = seq_lens, which
        include the token written above."""
        n = plan.n_dec
        pool = pool_for_layer(name, lay, query.device)
        ops.decode_paged(lay, cache, plan.block_size, md.block_table[:n], md.seq_lens[:n],
                         pool.decoders, plan.dec_rows(query.device), self._device_table(table, query),
                         query[:n], self.scale, output[:n], max(plan.seq_lens[:n]), images=pool.images)

    def _prefill(self, name, lay, cache, plan, md, table, query, key, value, output, skip_first=False):
        cont = []
        for r in plan.prefills:
            s, e = plan.qsl[r], plan.qsl[r + 1]
            if plan.seq_lens[r] < e - s:
                raise RuntimeError(
                    f"request {r} has seq_len={plan.seq_lens[r]} but {e - s} query tokens: the slot "
                    f"mapping and the sequence length disagree")
            if plan.seq_lens[r] == e - s:          # first chunk: its own post-RoPE q/k/v
                if not skip_first:                 # (else already attended on the side stream)
                    self._attend_first_chunks([r], plan, query, key, value, output)
            else:
                cont.append(r)
        if not cont:
            return
        dev = query.device
        pool = pool_for_layer(name, lay, dev)
        rows = [request_slot(plan.keys[r]) for r in cont]
        if any(x is None for x in rows):
            raise RuntimeError("a continuation chunk has no fitted decoder for its request")
        ridx = torch.tensor(cont, dtype=torch.long, device=dev)
        q_start = torch.tensor([plan.qsl[r] for r in cont], dtype=torch.int32, device=dev)
        q_len = torch.tensor([plan.qsl[r + 1] - plan.qsl[r] for r in cont], dtype=torch.int32, device=dev)
        ops.prefill_cont_paged(lay, cache, plan.block_size, md.block_table.index_select(0, ridx),
                               md.seq_lens.index_select(0, ridx), pool.decoders,
                               torch.tensor(rows, dtype=torch.int32, device=dev),
                               self._device_table(table, query), q_start, q_len, query, self.scale,
                               output, max(plan.qsl[r + 1] - plan.qsl[r] for r in cont),
                               max(plan.seq_lens[r] for r in cont), images=pool.images)

    # ------------------------------------------------------------------ resolution and guards
    @staticmethod
    def _device_table(table: torch.Tensor, query: torch.Tensor) -> torch.Tensor:
        if table.device != query.device:
            raise RuntimeError(f"the RoPE table is on {table.device}, the query on {query.device}")
        return table

    @staticmethod
    def _cos_sin_cache(layer, stash) -> torch.Tensor:
        """The model's own RoPE table (from the rotary capture, else `layer.rotary_emb`)."""
        csc = stash.get("cos_sin_cache")
        if csc is None:
            csc = getattr(getattr(layer, "rotary_emb", None), "cos_sin_cache", None)
        if csc is None:
            raise RuntimeError(
                f"layer {getattr(layer, 'layer_name', None)!r} has no RoPE table: the rotary capture "
                f"stashed none and `layer.rotary_emb.cos_sin_cache` is absent")
        return csc

    def _layout(self, layer) -> TTKLayout:
        lay = getattr(layer, "ttkv_layout", None)
        if lay is None:
            lay = layout_for_layer(getattr(layer, "layer_name", None))
        if lay is None:
            raise RuntimeError(
                f"no TT-KV layout for layer {getattr(layer, 'layer_name', None)!r}: load a calibration "
                f"table (VLLM_TTKV_CALIBRATION) or set `layer.ttkv_layout`")
        if lay.d != self.head_size:
            raise RuntimeError(
                f"the layout was built for head_dim={lay.d} but this layer has head_size={self.head_size}")
        return lay

    @staticmethod
    def _cache_tensor(kv_cache):
        if isinstance(kv_cache, (tuple, list)):
            raise RuntimeError(
                f"vllm_ttkv: expected ONE cache tensor (K and V share each slot) but got {len(kv_cache)}")
        return kv_cache

    @staticmethod
    def _block_size(cache) -> int:
        if cache.dim() == 4:                    # [num_blocks, head_slots, block_size, C]
            return int(cache.shape[2])
        if cache.dim() == 3:                    # [num_blocks, block_size, C]
            return int(cache.shape[1])
        raise ValueError(f"expected a page [num_blocks, head_slots, block_size, C], got {tuple(cache.shape)}")
