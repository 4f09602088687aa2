"""Paged TT-KV stores built entirely on the CPU by the oracle -- test infrastructure only.

A store built here exercises the CUDA read path independently of the CUDA write path: the bytes,
the block table, the decoders and the expected outputs all come from `ttkv_oracle`.
"""
from __future__ import annotations

import numpy as np

from oracle import ttkv_oracle as O
from vllm_ttkv import synthetic as S


def make_store(seed: int, seq_lens, cfg="safe", r1: int = 32, HQ: int = 24, H: int = 8,
               block_size: int = 16, dtype: str = "float16", ruler_div: str = "recip",
               extra_rows: int = 8):
    """A paged cache holding len(seq_lens) requests, each with its own fitted decoder.

    Returns a dict with numpy arrays: cache [n_slots, blob] uint8, block_table int32, seq_lens,
    decoders [B, r1, H*d] float32, pinvT [B, r1, H*d] float32, table [max_pos, 128] (float32
    values representable in `dtype`), q [B, HQ, 128], the geometry and per-request K/V.
    """
    g = O.geometry_for_config(cfg, r1, H=H)
    seq_lens = [int(n) for n in seq_lens]
    bt, n_blocks = S.block_table(seed, seq_lens, block_size)
    cache = np.zeros((n_blocks * block_size, g.blob_bytes), np.uint8)
    decoders = np.zeros((len(seq_lens), r1, H * 128), np.float32)
    pinvT = np.zeros_like(decoders)
    kv = []
    for r, n in enumerate(seq_lens):
        K, V = S.synth_kv(seed * 1000 + r, n, H=H)
        f = O.fit_into_budget(K, g, cfg, ruler_div)
        blobs = O.build_slots(g, f["coeff_q"], f["coeff_scale"], f["R"], V, ruler_div)
        cache[O.block_slots(bt[r], n, block_size)] = blobs
        decoders[r] = f["decoder_f"]
        pinvT[r] = np.linalg.pinv(f["decoder_f"]).T.astype(np.float32)
        kv.append((K, V))
    table = S.cos_sin_cache(max(seq_lens) + extra_rows, dtype=dtype)
    q = S.synth_queries(seed, (len(seq_lens), HQ, 128), dtype)
    return dict(g=g, cfg=cfg, cache=cache, block_table=bt, seq_lens=np.array(seq_lens, np.int32),
                decoders=decoders, pinvT=pinvT, table=table, q=q, kv=kv, block_size=block_size,
                dtype=dtype)


def expected_decode(st, q=None, scale=None):
    """Oracle decode over a store: [B, HQ, d] float32."""
    q = st["q"] if q is None else q
    return O.decode_batch(st["g"], st["cache"], st["block_table"], st["seq_lens"], st["block_size"],
                          q, list(st["decoders"]), st["table"], scale)


def expected_continuation(st, r: int, qm: np.ndarray, scale=None):
    """Oracle continuation for request r: qm [HQ, Q, d] at positions seq_len - Q + j."""
    g = st["g"]
    n = int(st["seq_lens"][r])
    slots = O.block_slots(st["block_table"][r], n, st["block_size"])
    ks, vs = O.read_blob(st["cache"], slots, g)
    cos, sin = O.cos_sin_from_table(st["table"], np.arange(n), g.d)
    Q = qm.shape[1]
    return O.attend_multi(g, ks, vs, st["decoders"][r], qm, cos, sin, scale, p0=n - Q)
