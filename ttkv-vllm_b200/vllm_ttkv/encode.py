"""The WRITE half: a step's raw K and V turned into packed slots in the paged cache.

Same two phases as the reference (vllm_ttkv/encode.py):

  * a request's FIRST chunk is fitted: TT-SVD of the [n, d, H] key block (tokens first), rank
    capped at the layer's budget and zero-padded to it (`fit_into_budget`, encode.py:257-298).
    The two decompositions stay library calls: `torch.linalg.svd` as in the reference, or, for a
    long chunk, the same subspaces from the eigendecomposition of the unfolding's Gram matrix
    (cuBLAS + cuSOLVER `eigh`, 6x faster at 1k and 16k tokens; `VLLM_TTKV_FIT`). Everything after them --
    coefficient/core quantisation, the decoder contraction, the decoder's own quantisation -- is
    `ops.fit_tail`, and the residual + V packing into the slots is `ops.write_paged` (fit path).
  * every later token is PROJECTED onto the request's frozen decoder (`encode_frozen`,
    encode.py:301-351): one `ops.write_paged` launch pair per layer for all requests, instead of
    ~20 torch launches per request.
"""
from __future__ import annotations

import os

import torch

from vllm_ttkv import ops
from vllm_ttkv.layout import TTKLayout, config


def active_config() -> dict:
    """The allocation named by VLLM_TTKV_CONFIG (default `safe`), as used for every fit."""
    import os
    return config(os.environ.get("VLLM_TTKV_CONFIG", "safe"))


def check_cfg_matches_layout(lay: TTKLayout, cfg: dict) -> None:
    """The layout must have been built from this allocation (vllm_ttkv/encode.py:103-135)."""
    want = dict(qbits=cfg["qbits"], res_k=max(int(lay.d * cfg["res_frac"]), 1),
                res_bits=cfg["res_bits"], v_lanes=cfg["k_lanes"], v_bits=cfg["vbits"])
    got = dict(qbits=lay.qbits, res_k=lay.res_k, res_bits=lay.res_bits, v_lanes=lay.v_lanes,
               v_bits=lay.v_bits)
    diff = {k: {"layout": got[k], "config": want[k]} for k in want if got[k] != want[k]}
    if diff:
        raise RuntimeError(
            f"the layout does not match the active allocation: {diff}. A store encoded under one "
            f"and read under the other has every field after the coefficients at the wrong offset.")


def as_kv_heads(x: torch.Tensor, H: int, d: int, what: str = "tensor") -> torch.Tensor:
    """`[T, H*d]` or `[T, H, d]` -> `[T, H, d]` (vllm_ttkv/encode.py:138-157)."""
    if x.dim() == 2:
        if x.shape[-1] != H * d:
            raise ValueError(f"{what} is [T, {x.shape[-1]}] but {H} kv heads of width {d} need {H * d}")
        return x.reshape(x.shape[0], H, d)
    if x.dim() == 3:
        if tuple(x.shape[1:]) != (H, d):
            raise ValueError(f"{what} is [T, {x.shape[1]}, {x.shape[2]}] but expected [T, {H}, {d}]")
        return x
    raise ValueError(f"{what} has {x.dim()} dims; expected 2 or 3")


class KDecoder:
    """A request's frozen decoder `[r1, H*d]` fp32 and the transposed pseudo-inverse the frozen
    projection needs (`[r1, H*d]`, i.e. pinv(decoder).T; computed once, vllm_ttkv/encode.py:178-211)."""

    __slots__ = ("decoder_f", "_pinvT")

    def __init__(self, decoder_f: torch.Tensor):
        if decoder_f.dim() != 2:
            raise ValueError(f"a decoder is [r1, H*d]; got {tuple(decoder_f.shape)}")
        self.decoder_f = decoder_f.float().contiguous()
        self._pinvT = None

    @property
    def pinv(self) -> torch.Tensor:
        return self.pinvT.t()

    @property
    def pinvT(self) -> torch.Tensor:
        if self._pinvT is None:
            self._pinvT = torch.linalg.pinv(self.decoder_f).t().contiguous()
        return self._pinvT

    def __repr__(self) -> str:
        return f"KDecoder(r1={self.decoder_f.shape[0]}, H*d={self.decoder_f.shape[1]})"


class FittedK:
    """The fit of one request's first chunk: codes, fp32 rulers (the residual is computed with
    the fp32 ruler; the slot stores it as fp16, codec/ttkv_packed_cache.py:353-375), the padded
    decoder and the quantised decoder it was built from."""

    __slots__ = ("coeff_q", "coeff_scale", "decoder", "dec_q", "dec_scale", "fitted_rank", "budget")

    def __init__(self, coeff_q, coeff_scale, decoder, dec_q, dec_scale, fitted_rank, budget):
        self.coeff_q, self.coeff_scale, self.decoder = coeff_q, coeff_scale, decoder
        self.dec_q, self.dec_scale = dec_q, dec_scale
        self.fitted_rank, self.budget = fitted_rank, budget

    def __repr__(self) -> str:
        return f"FittedK(rank {self.fitted_rank}/{self.budget}, {self.coeff_q.shape[0]} tokens)"


def _rank_from_spectrum(S: torch.Tensor, tol: float, cap: int | None) -> int:
    """Smallest rank whose dropped energy fraction is <= tol^2 (codec/ttkv_codec.py:96-103).
    One device readback per SVD, as in the reference."""
    e = S.pow(2)
    tail = torch.flip(torch.cumsum(torch.flip(e, [0]), 0), [0]) / (e.sum() + 1e-30)
    hit = torch.nonzero(tail <= tol ** 2, as_tuple=False)
    r = int(hit[0].item()) + 1 if hit.numel() else int(S.numel())
    r = max(1, min(r, int(S.numel())))
    return r if cap is None else max(1, min(r, cap))


FIT_ENV = "VLLM_TTKV_FIT"                 # "svd" | "gram" | "auto" (default)


def _svd_tall(X: torch.Tensor, method: str):
    """(S, Vh, U_of(r)) of a tall X [m, c]: the thin SVD's singular values (descending), right
    singular vectors, and a function giving the first r left singular vectors.

    "svd": torch.linalg.svd, as the reference (codec/ttkv_codec.py:96).
    "gram": the eigendecomposition of X^T X [c, c] (one GEMM and a c x c eigh): S = sqrt(lambda),
    Vh = the eigenvectors, U_r = X V_r / S_r. The same subspaces and singular values to fp32
    rounding of the Gram matrix; for the first unfolding of a 16384-token fit ([16384, 1024]) it
    took 12 ms on a B200 against 87 ms for the SVD. A direction with S = 0 gets a zero column."""
    if method == "svd":
        U, S, Vh = torch.linalg.svd(X, full_matrices=False)
        return S, Vh, lambda r: U[:, :r]
    lam, V = torch.linalg.eigh(X.T @ X)
    lam, V = lam.flip(0).clamp_min(0), V.flip(1)
    S = lam.sqrt()
    tiny = S.max() * 1e-7 if S.numel() else 0.0

    def left(r):
        inv = torch.where(S[:r] > tiny, 1.0 / S[:r].clamp_min(1e-30), torch.zeros_like(S[:r]))
        return (X @ V[:, :r]) * inv
    return S, V.T, left


GRAM_MIN_TOKENS = 256


def fit_method(n: int, width: int) -> str:
    """The first unfolding's decomposition: VLLM_TTKV_FIT, else "gram" from GRAM_MIN_TOKENS tokens
    on. A GPU SVD of an [n, width] unfolding costs far more than the eigendecomposition of its
    [width, width] Gram matrix once n is in the hundreds (70 ms against about 12 ms per layer at
    1082 x 1024 on a B200), and on the synthetic keys the two give the same ranks and
    reconstruction errors to 1e-6 relative from 256 to 16384 tokens (`tests/test_fit.py`)."""
    m = os.environ.get(FIT_ENV, "auto")
    if m not in ("svd", "gram", "auto"):
        raise ValueError(f"{FIT_ENV}={m!r}: expected svd, gram or auto")
    if m == "auto":
        return "gram" if n >= GRAM_MIN_TOKENS else "svd"
    return m


def tt_svd_cores(K: torch.Tensor, tol: float, max_rank: int | None, method: str | None = None):
    """TT-SVD of K [H, n, d] with tokens first ([n, d, H]): returns G1 [n, r], G2 [r, d, r2],
    G3 [r2, H] (codec/ttkv_codec.py:78-109 with the cores squeezed). `method` ("svd" or "gram",
    default `fit_method`) decomposes the first unfolding; the second, [r*d, H], always by Gram
    (H columns) unless "svd" is asked for."""
    H, n, d = K.shape
    X = K.permute(1, 2, 0).reshape(n, d * H).float()
    method = fit_method(n, d * H) if method is None else method
    S, Vh, left = _svd_tall(X, method)
    r = _rank_from_spectrum(S, tol, max_rank)
    G1 = left(r).contiguous()
    rest = (S[:r].unsqueeze(1) * Vh[:r, :]).reshape(r * d, H)
    S2, Vh2, left2 = _svd_tall(rest, "svd" if method == "svd" or r * d < 2 * H else "gram")
    r2 = _rank_from_spectrum(S2, tol, None)
    G2 = left2(r2).reshape(r, d, r2).contiguous()
    G3 = (S2[:r2].unsqueeze(1) * Vh2[:r2, :]).contiguous()
    return G1, G2, G3


def fit_into_budget(K: torch.Tensor, lay: TTKLayout, cfg: dict | str) -> FittedK:
    """A request's first chunk: K [H, n, d] (raw, any float dtype) -> FittedK at the layer's rank
    budget (vllm_ttkv/encode.py:257-298)."""
    cfg = config(cfg) if isinstance(cfg, str) else cfg
    check_cfg_matches_layout(lay, cfg)
    H, n, d = K.shape
    if (H, d) != (lay.H, lay.d):
        raise ValueError(f"K is [H={H}, n={n}, d={d}] but the layout is for H={lay.H}, d={lay.d}")
    G1, G2, G3 = tt_svd_cores(K.float(), cfg["tols"], lay.r1)
    out = ops.fit_tail(G1, G2, G3, lay.r1, cfg["qbits"])
    return FittedK(out["coeff_q"], out["coeff_scale"], KDecoder(out["decoder"]), out["dec_q"],
                   out["dec_scale"], int(G1.shape[1]), lay.r1)


def write_fitted(cache_u8: torch.Tensor, slot_mapping: torch.Tensor, fk: FittedK, K_tok, V_tok,
                 lay: TTKLayout, pool_index: torch.Tensor | None = None,
                 heads: tuple[int, int] | None = None) -> None:
    """Write a fitted chunk: K_tok / V_tok [n, H, d], slot ids [n] int64. heads: the KV heads a
    storage-sharded cache holds (rows of `lay.shard(*heads)`)."""
    n = slot_mapping.numel()
    dec = fk.decoder.decoder_f.unsqueeze(0)
    tok_dec = torch.zeros(n, dtype=torch.int32, device=K_tok.device) if pool_index is None else pool_index
    ops.write_paged(lay, cache_u8, slot_mapping, K_tok, V_tok, tok_dec, dec,
                    coeff_q=fk.coeff_q, coeff_scale=fk.coeff_scale, heads=heads)


def write_frozen(cache_u8: torch.Tensor, slot_mapping: torch.Tensor, K_tok, V_tok,
                 tok_dec: torch.Tensor, decoders: torch.Tensor, pinvT: torch.Tensor,
                 lay: TTKLayout, skip_pad: bool = False, heads: tuple[int, int] | None = None) -> None:
    """Project every token onto its request's frozen decoder and write it (one launch for the
    whole layer): K_tok / V_tok [n, H, d]; tok_dec [n] index into the decoder pool. skip_pad:
    padding tokens (PAD_SLOT_ID) are skipped rather than refused. heads: the KV heads a
    storage-sharded cache holds (rows of `lay.shard(*heads)`)."""
    ops.write_paged(lay, cache_u8, slot_mapping, K_tok, V_tok, tok_dec, decoders, pinvs=pinvT,
                    skip_pad=skip_pad, heads=heads)
