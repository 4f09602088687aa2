"""Registries shared by the backend, the writer and the reader.

Same surface as the reference's `vllm_ttkv/rope_store.py`:
  * the calibration table -> per-layer `TTKLayout` (load_calibration, layout_for_layer);
  * the live per-layer store holding the model's RoPE table (TTKVRopeStore, ensure_store);
  * the per-(layer, request) decoder registry keyed by the request's first block
    (register_decoder, decoder_for_request, release_decoder, clear_decoders).

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
import re

import torch

from vllm_ttkv import ops
from vllm_ttkv.layout import TTKLayout, config, layout_for_config

CONFIG_ENV = "VLLM_TTKV_CONFIG"
CALIBRATION_ENV = "VLLM_TTKV_CALIBRATION"

_STORES: dict[str, "TTKVRopeStore"] = {}
_CALIBRATED: dict[int, TTKLayout] = {}
_CALIBRATION: dict = {}
_DECODERS: dict[tuple[str, int], "object"] = {}       # (layer, key) -> KDecoder
_POOLS: dict[str, "DecoderPool"] = {}
_REQ_SLOT: dict[int, int] = {}                         # request key -> pool row (all layers)
_FREE_SLOTS: list[int] = []
_NEXT_SLOT = [0]


def _layer_index(layer_name: str) -> int | None:
    m = re.search(r"layers\.(\d+)", layer_name)
    if m:
        return int(m.group(1))
    nums = re.findall(r"(\d+)", layer_name)
    return int(nums[-1]) if nums else None


def load_calibration(path, cfg_name: str = "safe", cfg: dict | None = None) -> dict:
    """Per-layer layouts from a calibration artifact with keys r1, layers, heads, head_dim
    (the reference's tools/calibrate_r1.py format, rope_store.py:70-103)."""
    global _CALIBRATION
    cfg = config(cfg_name) if cfg is None else cfg
    data = json.loads(pathlib.Path(path).read_text())
    r1 = data["r1"]
    if len(r1) != data["layers"]:
        raise ValueError(f"{path}: r1 has {len(r1)} entries but layers={data['layers']}")
    _CALIBRATED.clear()
    for idx, rank in enumerate(r1):
        _CALIBRATED[idx] = layout_for_config(cfg, int(rank), H=data["heads"], d=data["head_dim"])
    _CALIBRATION = dict(data)
    return _CALIBRATION


def calibration_info() -> dict:
    return dict(_CALIBRATION)


def layout_for_layer(layer_name: str | None) -> TTKLayout | None:
    if layer_name is None:
        return None
    store = _STORES.get(layer_name)
    if store is not None:
        return store.layout
    idx = _layer_index(layer_name)
    return _CALIBRATED.get(idx) if idx is not None else None


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


class DecoderPool:
    """One layer's device decoders `[cap, r1, H*d]` fp32, their transposed pseudo-inverses, and
    the decode's operand images of them (`ops.decoder_image`, made once per decoder)."""

    def __init__(self, lay: TTKLayout, device, capacity: int = 16):
        self.lay, self.device = lay, torch.device(device)
        self.decoders = torch.zeros(capacity, lay.r1, lay.H * lay.d, device=self.device)
        self.pinvT = torch.zeros_like(self.decoders)
        # None: a host pool, or a layout the tensor-core decode does not serve
        self.images = ops.decoder_image(lay, self.decoders) if self.device.type == "cuda" else None

    @property
    def capacity(self) -> int:
        return self.decoders.shape[0]

    def _grow(self, need: int):
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
        pool = DecoderPool(lay, device)
        _POOLS[layer_name] = pool
    return pool


def register_decoder(layer_name: str, key: int, decoder, lay: TTKLayout | None = None) -> None:
    """Publish a request's fitted decoder for this layer (host registry + device pool); `lay` is the
    layer's layout when it does not come from the calibration table."""
    _DECODERS[(layer_name, key)] = decoder
    lay = lay if lay is not None else layout_for_layer(layer_name)
    if lay is not None and decoder.decoder_f.is_cuda:
        slot = request_slot(key, create=True)
        pool_for_layer(layer_name, lay, decoder.decoder_f.device).put(slot, decoder)


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


def release_request(key: int) -> None:
    for name in [n for (n, k) in _DECODERS if k == key]:
        release_decoder(name, key)


def clear_decoders() -> None:
    _DECODERS.clear()
    _POOLS.clear()
    _REQ_SLOT.clear()
    _FREE_SLOTS.clear()
    _NEXT_SLOT[0] = 0


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
