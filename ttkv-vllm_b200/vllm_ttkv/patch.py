"""The raw (pre-RoPE) key hand-over between a model's rotary call and the TT-KV attention impl.

The store holds keys BEFORE rotation (the position-free keys are what the tensor-train fit
compresses), but a model rotates q and k before it calls attention. So the key is captured at the
model's own rotary call, `q, k = self.rotary_emb(positions, q, k)`, which receives raw k, and handed
to the attention impl of the same layer in the same forward (vllm_ttkv/patch.py:253-263 in the
reference).

* `stash_raw_k(layer, raw_k, positions, cos_sin_cache)` records the capture; `take_raw_k(layer)`
  POPS it, so a second consumer in the same step raises instead of re-reading a stale key.
* `RawKCapture(rotary, layer_name)` wraps a rotary module: it stashes the key it is called with,
  then runs the wrapped module unchanged.
* `install(model)` wraps the rotary module of every attention block whose attention layer has a
  `layer_name`, and raises when it wraps nothing (a silent miss would store post-RoPE keys).
"""
from __future__ import annotations

from torch import nn

_RAW_K_STASH: dict[str, dict] = {}


def stash_raw_k(layer_name: str, raw_k, positions, cos_sin_cache=None) -> None:
    if layer_name in _RAW_K_STASH:
        raise RuntimeError(
            f"vllm_ttkv: a raw key for layer {layer_name!r} is already waiting: the previous "
            f"capture was never consumed by the attention impl, so that step wrote no store.")
    _RAW_K_STASH[layer_name] = {"raw_k": raw_k, "positions": positions, "cos_sin_cache": cos_sin_cache}


def take_raw_k(layer_name: str) -> dict:
    """Pop this layer's capture; raise if the rotary wrapper did not run first."""
    try:
        return _RAW_K_STASH.pop(layer_name)
    except KeyError:
        raise RuntimeError(
            f"vllm_ttkv: no raw K stashed for layer {layer_name!r}. The rotary wrapper did not run "
            f"before attention, so the store would receive post-RoPE keys. Refusing.") from None


def clear_stash() -> None:
    _RAW_K_STASH.clear()


class RawKCapture(nn.Module):
    """Wraps a rotary module: stashes the raw key of each call under `layer_name`, then rotates."""

    def __init__(self, inner: nn.Module, layer_name: str):
        super().__init__()
        # kept out of the module tree, so the wrapped module's parameter and buffer names (the
        # checkpoint's names) stay what they were
        object.__setattr__(self, "_inner", inner)
        self._ttkv_layer_name = layer_name

    def __getattr__(self, item):
        if item == "_inner":
            raise AttributeError(item)
        return getattr(self._inner, item)

    def forward(self, positions, query, key=None, *args, **kwargs):
        raw_k = key if key is not None else kwargs.get("key")
        if raw_k is None:
            raise RuntimeError(
                "vllm_ttkv: the rotary module was called without a key, so the raw key cannot be "
                "captured for the store.")
        stash_raw_k(self._ttkv_layer_name, raw_k, positions, getattr(self._inner, "cos_sin_cache", None))
        return self._inner(positions, query, key, *args, **kwargs)


def install(model: nn.Module, attn_attr: str = "attn", rotary_attr: str = "rotary_emb") -> int:
    """Wrap the rotary module of every block that owns both `rotary_attr` and an attention layer
    `attn_attr` carrying a `layer_name`. Returns the number of layers wrapped."""
    n = 0
    for mod in model.modules():
        rot = getattr(mod, rotary_attr, None)
        attn = getattr(mod, attn_attr, None)
        name = getattr(attn, "layer_name", None)
        if rot is None or name is None or isinstance(rot, RawKCapture):
            continue
        setattr(mod, rotary_attr, RawKCapture(rot, name))
        n += 1
    if n == 0:
        raise RuntimeError(
            f"vllm_ttkv: found no block with both `.{rotary_attr}` and `.{attn_attr}.layer_name`, "
            f"so no raw key would be captured and the store would receive post-RoPE keys.")
    return n
