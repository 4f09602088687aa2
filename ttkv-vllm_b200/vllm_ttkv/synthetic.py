"""Seeded synthetic inputs for the TT-KV hot path (benchmark and test workloads).

Self-contained numpy: no other `vllm_ttkv` module is imported, so a script can load this file by
path next to another package of the same name.

The reference measures on real Llama-3.2-3B activations (RULER / LongBench prose); neither the
weights nor the datasets exist here, so these generators stand in with the same SHAPES and a key
distribution that has the property the codec exploits (low rank across tokens):

    K_h = Z_h @ B_h + E_h   per KV head,  Z ~ N(0,1) [n, 96],  B ~ N(0, 1/96) [96, d],
                            4 outlier channels per head with their B columns scaled x8,
                            E ~ 0.02 * N(0,1)
    V ~ N(0,1),  q ~ N(0,1) (post-RoPE, as the model hands it to attention)

RoPE is Llama-3.2-3B's: theta 500000 with llama3 frequency scaling (factor 32, low 1, high 4,
original context 8192), laid out as vLLM's `cos_sin_cache` = cat(cos, sin) and cast to the model
dtype, because the model's table is what the query was rotated with.
"""
from __future__ import annotations

import math

import numpy as np

# Per-layer TT rank budget of Llama-3.2-3B at tol 0.2 and 16k context, from the reference's
# calibration artifact `calibration/llama-3.2-3b-16384.json` (key "r1"; per-layer max over its
# corpus samples). It is an input to the format -- it sizes each layer's slot -- not code.
LLAMA32_3B_R1 = [14, 28, 143, 105, 74, 130, 108, 86, 107, 110, 117, 77, 118, 117, 115, 107, 116,
                 122, 125, 104, 111, 108, 119, 105, 134, 138, 82, 67]

LLAMA32_3B = dict(layers=28, hidden=3072, num_heads=24, num_kv_heads=8, head_dim=128,
                  rope_theta=500000.0, rope_factor=32.0, low_freq_factor=1.0,
                  high_freq_factor=4.0, original_max_position=8192)


def synth_kv(seed: int, n: int, H: int = 8, d: int = 128, rank: int = 96, n_outliers: int = 4,
             noise: float = 0.02):
    """(K, V) each [H, n, d] float32. Deterministic for a given numpy build and CPU."""
    rng = np.random.default_rng(seed)
    K = np.empty((H, n, d), np.float32)
    for h in range(H):
        Z = rng.standard_normal((n, rank), dtype=np.float32)
        B = (rng.standard_normal((rank, d), dtype=np.float32) * np.float32(1.0 / math.sqrt(rank)))
        ch = rng.choice(d, n_outliers, replace=False)
        B[:, ch] *= np.float32(8.0)
        E = rng.standard_normal((n, d), dtype=np.float32) * np.float32(noise)
        K[h] = Z @ B + E
    V = rng.standard_normal((H, n, d), dtype=np.float32)
    return K, V


def synth_queries(seed: int, shape, dtype=np.float16):
    """Post-RoPE queries ~ N(0,1), rounded to the model dtype (fp16/bf16 via float32 bits)."""
    rng = np.random.default_rng(seed + 7919)
    q = rng.standard_normal(shape, dtype=np.float32)
    return round_to_dtype(q, dtype)


def round_to_dtype(x: np.ndarray, dtype) -> np.ndarray:
    """float32 array with values representable in `dtype` ("float16"/"bfloat16"/"float32")."""
    name = np.dtype(dtype).name if not isinstance(dtype, str) else dtype
    if name in ("float32",):
        return x.astype(np.float32)
    if name in ("float16",):
        return x.astype(np.float16).astype(np.float32)
    if name in ("bfloat16",):
        u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16          # round to nearest even
        return r.astype(np.uint32).view(np.float32)
    raise ValueError(dtype)


def llama3_inv_freq(d: int = 128, theta: float = 500000.0, factor: float = 32.0,
                    low: float = 1.0, high: float = 4.0, old: int = 8192) -> np.ndarray:
    """The llama3-scaled RoPE frequencies (Llama 3.1+ `rope_scaling` "llama3")."""
    inv = (1.0 / (np.float32(theta) ** (np.arange(0, d, 2, dtype=np.float32) / np.float32(d))))
    inv = inv.astype(np.float32)
    wl = (2 * math.pi / inv).astype(np.float32)
    lw, hw = old / low, old / high
    smooth = ((old / wl - low) / (high - low)).astype(np.float32)
    scaled = np.where(wl > lw, inv / factor, (1 - smooth) * inv / factor + smooth * inv)
    return np.where(wl < hw, inv, scaled).astype(np.float32)


def cos_sin_cache(max_pos: int, d: int = 128, dtype="float16", **rope) -> np.ndarray:
    """vLLM's `RotaryEmbedding.cos_sin_cache` layout: [max_pos, d] = cat(cos, sin), values
    rounded to the model dtype and returned as float32 (the kernels read the 16-bit bits)."""
    inv = llama3_inv_freq(d, **rope)
    f = np.outer(np.arange(max_pos, dtype=np.float32), inv).astype(np.float32)
    table = np.concatenate([np.cos(f), np.sin(f)], axis=-1).astype(np.float32)
    return round_to_dtype(table, dtype)


def to_bits16(x: np.ndarray, dtype) -> np.ndarray:
    """uint16 bit patterns of a float32 array already rounded to fp16 / bf16."""
    name = dtype if isinstance(dtype, str) else np.dtype(dtype).name
    if name == "float16":
        return x.astype(np.float16).view(np.uint16)
    if name == "bfloat16":
        return (round_to_dtype(x, "bfloat16").view(np.uint32) >> 16).astype(np.uint16)
    raise ValueError(dtype)


def block_table(seed: int, seq_lens, block_size: int = 16, spare_blocks: int = 3):
    """A non-contiguous block table: every request's blocks drawn from one seeded permutation of
    the pool (as vLLM's allocator hands them out after churn), padded with -1 past each row's used
    prefix. Returns (table int32 [B, max_blocks], n_blocks_total)."""
    need = [-(-int(n) // block_size) for n in seq_lens]
    total = sum(need) + spare_blocks
    perm = np.random.default_rng(seed + 104729).permutation(total).astype(np.int32)
    width = max(need) if need else 1
    bt = np.full((len(seq_lens), max(width, 1)), -1, np.int32)
    at = 0
    for r, k in enumerate(need):
        bt[r, :k] = perm[at:at + k]
        at += k
    return bt, total
