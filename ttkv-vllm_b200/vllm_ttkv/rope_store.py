"""Registries shared by the backend, the writer and the reader.

Same surface as the reference's `vllm_ttkv/rope_store.py`:
  * the calibration table -> per-layer `TTKLayout` (load_calibration, layout_for_layer);
  * the live per-layer store holding the model's RoPE table (TTKVRopeStore, ensure_store);
  * the per-(layer, request) decoder registry keyed by the request's first block
    (register_decoder, decoder_for_request, release_decoder, clear_decoders).

Graph capture. A decode step can be planned without reading anything back (`rows_for_keys` maps
each request's key to its pool row on the device). A CUDA graph captured over it holds the raw
addresses of the pools and of the key map, so those are `pin`ned by the capture: they stay alive
for the process, and a pinned pool or key map refuses to grow (size them first with
`reserve_rows` / `reserve_keys`).

What changes is where decoders live. The reference keeps a host dict of fp32 tensors, one lookup
per request per layer (rope_store.py:169-237), which a batched kernel cannot read. Here every
registered decoder also occupies a row of a per-layer DEVICE pool (`DecoderPool`), and a request
keeps the SAME row index in every layer (`request_slot`), so one int32 vector per step tells
every layer's read and write kernel where each request's decoder is. `release_decoder` frees the
row (the reference's release is never called, rope_store.py:230).
"""
from __future__ import annotations

import json
import pathlib

import torch

from vllm_ttkv import ops
from vllm_ttkv.layout import TTKLayout, config, layout_for_config

CONFIG_ENV = "VLLM_TTKV_CONFIG"
CALIBRATION_ENV = "VLLM_TTKV_CALIBRATION"

_STORES: dict[str, "TTKVRopeStore"] = {}
_DECODERS: dict[tuple[str, int], "object"] = {}       # (layer, key) -> KDecoder
_POOLS: dict[str, "DecoderPool"] = {}
_REQ_SLOT: dict[int, int] = {}                         # request key -> pool row (all layers)
_FREE_SLOTS: list[int] = []
_NEXT_SLOT = [0]
_KEY_ROWS: dict[torch.device, torch.Tensor] = {}       # device copy of _REQ_SLOT: key -> row, -1
_RESERVE = [16]                                        # pool rows a new pool starts with


class Calibration:
    """A loaded per-layer rank table: the artifact as read (its metadata travels with any slot
    size derived from it) and the layout each transformer block gets from it.

    The artifact is the reference's calibration JSON (keys `r1` = one rank per block, `layers`,
    `heads`, `head_dim`, plus free-form provenance such as the corpus; rope_store.py:70-103 reads
    the same keys). Layouts are built once at load time, so a lookup is a list index."""

    def __init__(self, data: dict, cfg: dict, source: str = "<dict>"):
        ranks = [int(x) for x in data["r1"]]
        if len(ranks) != int(data["layers"]):
            raise ValueError(f"{source}: calibration lists {len(ranks)} ranks (r1) for "
                             f"{data['layers']} layers")
        self.meta = dict(data)
        self.layouts = [layout_for_config(cfg, r, H=int(data["heads"]), d=int(data["head_dim"]))
                        for r in ranks]

    def layout(self, block: int | None) -> TTKLayout | None:
        if block is None or not 0 <= block < len(self.layouts):
            return None
        return self.layouts[block]


_CAL: list[Calibration] = []                             # the loaded table (at most one)


def block_index(layer_name: str) -> int | None:
    """The transformer block a vLLM layer name belongs to: the integer component that follows a
    `layers` component (`model.layers.7.self_attn.attn` -> 7); failing that, the last all-digit
    component (a spec may carry a shortened name such as `attn.7`); None when there is none.
    A name that resolves to no block is reported as uncalibrated by the lookup, never guessed."""
    parts = layer_name.split(".")
    for prev, cur in zip(parts, parts[1:]):
        if prev == "layers" and cur.isdigit():
            return int(cur)
    digits = [p for p in parts if p.isdigit()]
    return int(digits[-1]) if digits else None


def load_calibration(path, cfg_name: str = "safe", cfg: dict | None = None) -> dict:
    """Load a calibration artifact (see `Calibration`) under allocation `cfg` (default: the
    named one) and make it the table `layout_for_layer` falls back to. Returns its metadata."""
    cal = Calibration(json.loads(pathlib.Path(path).read_text()),
                      config(cfg_name) if cfg is None else cfg, source=str(path))
    _CAL[:] = [cal]
    return dict(cal.meta)


def calibration_info() -> dict:
    """The loaded artifact's metadata, or {} when no table is loaded."""
    return dict(_CAL[0].meta) if _CAL else {}


def layout_for_layer(layer_name: str | None) -> TTKLayout | None:
    """A layer's layout. A live store (one exists once a forward has fitted the layer) is the
    truth; before any forward (cache sizing) only the calibration table can answer. None means
    the layer cannot be served; callers raise."""
    if layer_name is None:
        return None
    live = _STORES.get(layer_name)
    if live is not None:
        return live.layout
    if not _CAL:
        return None
    return _CAL[0].layout(block_index(layer_name))


# ------------------------------------------------------------------ request keys
def request_key_host(row) -> int:
    """A request's identity: its first physical block (rope_store.py:180-207)."""
    if not len(row):
        raise ValueError("the block table row is empty, so this request has no blocks and no "
                         "identity to key a decoder by")
    return int(row[0])


def request_key(block_row: torch.Tensor) -> int:
    if block_row.numel() == 0:
        raise ValueError("the block table row is empty, so this request has no blocks and no "
                         "identity to key a decoder by")
    return int(block_row[0])


def request_slot(key: int, create: bool = False) -> int | None:
    """The pool row a request uses in every layer (assigned on its first registration)."""
    s = _REQ_SLOT.get(key)
    if s is None and create:
        s = _FREE_SLOTS.pop() if _FREE_SLOTS else _NEXT_SLOT[0]
        if s == _NEXT_SLOT[0]:
            _NEXT_SLOT[0] += 1
        _REQ_SLOT[key] = s
    return s


# ------------------------------------------------------------------ the device key map
def key_rows(device, n_keys: int = 0) -> torch.Tensor:
    """The device's key -> pool row map (int32, -1 where a key has no row), holding at least
    `n_keys` keys (a request's key is a block id, so the cache's block count covers every key)."""
    dev = torch.device(device)
    lut = _KEY_ROWS.get(dev)
    if lut is None or lut.numel() < n_keys:
        if ops.capturing():
            # made inside a capture, its initialisation would be a node that every replay reruns
            raise RuntimeError(
                f"the decoder key map on {dev} must hold {n_keys} keys before a CUDA graph capture: "
                f"run one eager step first or call rope_store.reserve_keys")
        if lut is not None and ops.is_pinned(lut):
            raise RuntimeError(
                f"the decoder key map on {dev} holds {lut.numel()} keys and a captured CUDA graph "
                f"reads it, so it cannot grow to {n_keys}; call rope_store.reserve_keys before the "
                f"capture")
        n = max(1024, n_keys, 0 if lut is None else lut.numel(), max(_REQ_SLOT, default=-1) + 1)
        new = torch.full((n,), -1, dtype=torch.int32, device=dev)
        if lut is not None:
            new[:lut.numel()] = lut
        else:
            for key, row in _REQ_SLOT.items():
                if key < n:
                    new[key] = row
        lut = new
        _KEY_ROWS[dev] = lut
    return lut


def reserve_keys(n_keys: int, device) -> torch.Tensor:
    """Size the device key map for block ids below `n_keys` (before a graph capture)."""
    return key_rows(device, n_keys)


def rows_for_keys(keys: torch.Tensor) -> torch.Tensor:
    """Pool rows (int32, -1 for a key without a decoder) of device request keys, on the device:
    no readback, so a decode step planned with it can be captured in a CUDA graph. A key outside
    the map reads -1 (the kernels then refuse the request on the device)."""
    lut = key_rows(keys.device)
    k = keys.to(torch.int64)
    ok = (k >= 0) & (k < lut.numel())
    rows = lut.index_select(0, k.clamp(0, lut.numel() - 1))
    return torch.where(ok, rows, torch.full_like(rows, -1))


def _set_key_row(key: int, row: int) -> None:
    for dev, lut in _KEY_ROWS.items():
        if key >= lut.numel():
            lut = key_rows(dev, max(key + 1, 2 * lut.numel()))
        lut[key] = row


def reserve_rows(n_rows: int) -> None:
    """Give every decoder pool (existing and later) at least `n_rows` rows, e.g. the engine's
    maximum number of live requests, so that no pool has to grow after a graph capture."""
    _RESERVE[0] = max(_RESERVE[0], int(n_rows))
    for pool in _POOLS.values():
        if pool.capacity < n_rows:
            pool._grow(n_rows - 1)


class DecoderPool:
    """One layer's device decoders `[cap, r1, H*d]` fp32, their transposed pseudo-inverses, and
    the decode's operand images of them (`ops.decoder_image`, made once per decoder)."""

    def __init__(self, lay: TTKLayout, device, capacity: int | None = None):
        self.lay, self.device = lay, torch.device(device)
        capacity = _RESERVE[0] if capacity is None else capacity
        self.decoders = torch.zeros(capacity, lay.r1, lay.H * lay.d, device=self.device)
        self.pinvT = torch.zeros_like(self.decoders)
        # None: a host pool, or a layout the tensor-core decode does not serve
        self.images = ops.decoder_image(lay, self.decoders) if self.device.type == "cuda" else None

    @property
    def capacity(self) -> int:
        return self.decoders.shape[0]

    def pin(self) -> None:
        """Keep this pool's tensors alive and fixed: a captured CUDA graph reads them."""
        ops.pin(self.decoders, self.pinvT, *(self.images or ()))

    def _grow(self, need: int):
        if ops.is_pinned(self.decoders):
            raise RuntimeError(
                f"the decoder pool holds {self.capacity} rows and a captured CUDA graph reads it, so "
                f"it cannot grow to row {need}; call rope_store.reserve_rows before the capture")
        cap = self.capacity
        while cap <= need:
            cap *= 2
        dec = torch.zeros(cap, *self.decoders.shape[1:], device=self.device)
        pin = torch.zeros_like(dec)
        dec[:self.capacity] = self.decoders
        pin[:self.capacity] = self.pinvT
        self.decoders, self.pinvT = dec, pin
        if self.images is not None:
            self.images = ops.decoder_image(self.lay, self.decoders)

    def put(self, slot: int, kdec) -> None:
        if slot >= self.capacity:
            self._grow(slot)
        self.decoders[slot] = kdec.decoder_f
        self.pinvT[slot] = kdec.pinvT
        if self.images is not None:
            image, scales = self.images
            ops.decoder_image(self.lay, self.decoders[slot:slot + 1],
                              out=(image[slot:slot + 1], scales[slot:slot + 1]))


def pool_for_layer(layer_name: str, lay: TTKLayout, device) -> DecoderPool:
    pool = _POOLS.get(layer_name)
    if pool is None or pool.lay.r1 != lay.r1 or pool.device != torch.device(device):
        if ops.capturing():
            raise RuntimeError(
                f"layer {layer_name!r} has no decoder pool and one cannot be made inside a CUDA "
                f"graph capture (its zero fill would rerun at every replay): run one eager step "
                f"first")
        pool = DecoderPool(lay, device)
        _POOLS[layer_name] = pool
    return pool


def register_decoder(layer_name: str, key: int, decoder, lay: TTKLayout | None = None) -> None:
    """Publish a request's fitted decoder for this layer (host registry + device pool); `lay` is the
    layer's layout when it does not come from the calibration table."""
    _DECODERS[(layer_name, key)] = decoder
    lay = lay if lay is not None else layout_for_layer(layer_name)
    if lay is not None and decoder.decoder_f.is_cuda:
        fresh = key not in _REQ_SLOT
        slot = request_slot(key, create=True)
        pool_for_layer(layer_name, lay, decoder.decoder_f.device).put(slot, decoder)
        if fresh:
            key_rows(decoder.decoder_f.device, key + 1)
            _set_key_row(key, slot)


def decoder_for_request(layer_name: str | None, key: int):
    if layer_name is None:
        return None
    return _DECODERS.get((layer_name, key))


def release_decoder(layer_name: str, key: int) -> None:
    """Drop a finished request's decoder for this layer; the pool row is returned when the
    request holds no decoder in any layer."""
    _DECODERS.pop((layer_name, key), None)
    if not any(k == key for (_, k) in _DECODERS):
        s = _REQ_SLOT.pop(key, None)
        if s is not None:
            _FREE_SLOTS.append(s)
            _set_key_row(key, -1)


def release_request(key: int) -> None:
    """Drop a finished request's decoder in every layer and return its pool row (the next
    registered request takes it over). The engine calls this when the request completes; the
    reference never releases (rope_store.py:230), so its registry grows for the whole run."""
    for name in [n for (n, k) in _DECODERS if k == key]:
        release_decoder(name, key)
    s = _REQ_SLOT.pop(key, None)               # a key registered with no layer left (defensive)
    if s is not None:
        _FREE_SLOTS.append(s)
        _set_key_row(key, -1)


def live_keys() -> set[int]:
    """Keys (first block ids) of the requests holding a decoder pool row."""
    return set(_REQ_SLOT)


def pool_rows_in_use() -> int:
    return len(_REQ_SLOT)


class AbsenceReaper:
    """Releases requests that no step has named for `after` consecutive steps: a fallback for an
    engine that does not report completions. A request that merely sits out steps (a prefill
    chunk held back by the token budget, another pipeline micro-batch) must not be released, so
    `after` has to exceed the longest such gap; off (0) unless VLLM_TTKV_RELEASE_AFTER is set."""

    def __init__(self, after: int):
        self.after = int(after)
        self._missed: dict[int, int] = {}

    def step(self, keys) -> list[int]:
        """Record the keys of a step's requests; returns the keys released by this call."""
        if self.after <= 0:
            return []
        seen = {int(k) for k in keys}
        released = []
        for k in list(_REQ_SLOT):
            if k in seen:
                self._missed.pop(k, None)
                continue
            n = self._missed.get(k, 0) + 1
            if n >= self.after:
                release_request(k)
                self._missed.pop(k, None)
                released.append(k)
            else:
                self._missed[k] = n
        return released


def clear_decoders() -> None:
    """Forget every decoder. A pinned key map is kept (emptied), so a graph that reads it sees no
    request; a pinned pool stays alive but is no longer the layer's pool."""
    _DECODERS.clear()
    _POOLS.clear()
    _REQ_SLOT.clear()
    _FREE_SLOTS.clear()
    _NEXT_SLOT[0] = 0
    for dev in list(_KEY_ROWS):
        if ops.is_pinned(_KEY_ROWS[dev]):
            _KEY_ROWS[dev].fill_(-1)
        else:
            del _KEY_ROWS[dev]


def decoder_for_layer(layer_name: str | None):
    store = _STORES.get(layer_name) if layer_name else None
    return None if store is None else store.decoder_f


class TTKVRopeStore:
    """Holds the model's RoPE table for a layer (rope_store.py:240-278)."""

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int,
                 cos_sin_cache: torch.Tensor, layer_name: str, layout: TTKLayout):
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.cos_sin_cache = cos_sin_cache
        self.layer_name, self.layout = layer_name, layout
        self.decoder_f = None
        _STORES[layer_name] = self


def ensure_store(layer_name: str, cos_sin_cache: torch.Tensor, num_heads: int, num_kv_heads: int,
                 head_dim: int, layout: TTKLayout | None) -> TTKVRopeStore:
    store = _STORES.get(layer_name)
    if store is not None:
        return store
    if layout is None:
        raise RuntimeError(
            f"cannot create a TT-KV store for layer {layer_name!r}: no calibrated layout. Point "
            f"{CALIBRATION_ENV} at a calibration artifact.")
    return TTKVRopeStore(num_heads, num_kv_heads, head_dim, cos_sin_cache, layer_name, layout)


def store_for_layer(layer_name: str | None) -> TTKVRopeStore | None:
    return _STORES.get(layer_name) if layer_name else None


def clear_stores() -> None:
    _STORES.clear()
