"""CPU restatement of the TT-KV compressed-KV attention path -- TEST INFRASTRUCTURE ONLY.

This module is the CHECKER for the CUDA path, never part of it. Only `tests/`,
`__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm may import it. The product
(`vllm_ttkv` + `libttkv_sm100.so`) never calls into this file and has no CPU fallback.

It restates, in numpy, the reference's algorithm for the hot path (Yaweni/ttkv-vllm; every
function names the reference file:line it follows):

  * the slot geometry and byte format     vllm_ttkv/layout.py, codec/ttkv_packed_cache.py
  * the quantisers (rulers, codes, masks) codec/ttkv_packed_cache.py, codec/ttkv_codec.py
  * the fit tail and frozen projection    vllm_ttkv/encode.py, codec/ttkv_packed_cache.py
  * the decode / continuation read        vllm_ttkv/reference.py, vllm_ttkv/decode.py

Two spellings of one rule are carried explicitly, because the reference itself has both:
`ruler_div` selects how a ruler is divided by the Python-int divisor `2**(bits-1)-1`.
  - "recip": multiply by the fp32 reciprocal. This is what torch's CUDA kernel does for
    `tensor / python_scalar` and what the reference's fused writer reproduces on purpose
    (vllm_ttkv/select_triton.py:76-84, :119). It is the serving path's format, so it is the
    default and what the CUDA kernels match.
  - "true": a correctly rounded division, which is what torch's CPU kernel does for the same
    expression. The reference run on CPU (how the golden vectors are generated) uses this one.

Parity pinning: `tests/golden/make_golden.py` imports the reference from its source tree, runs it
on seeded inputs (plain, and with the CUDA division rule emulated) and stores the outputs; the
`-m "not gpu"` tests check every function here against those vectors.
"""
from __future__ import annotations

import math

import numpy as np

# ----------------------------------------------------------------------------- configs
# The three allocations of codec/ttkv_codec.py:272-298. These are format parameters (they decide
# slot widths), so the numbers must be the reference's.
CONFIGS = {
    "safe": dict(tols=0.20, qbits=8, res_frac=0.633, res_bits=3, k_lanes=81, vbits=3),
    "tight": dict(tols=0.20, qbits=8, res_frac=0.25, res_bits=3, k_lanes=45, vbits=3),
    "campaign4x": dict(tols=0.20, qbits=8, res_frac=0.50, res_bits=4, k_lanes=64, vbits=4),
}


# ----------------------------------------------------------------------------- geometry
def align_up(n: int, a: int) -> int:
    """vllm_ttkv/layout.py:44-47."""
    return n if a <= 1 else ((n + a - 1) // a) * a


def packed_row_bytes(k: int, bits: int) -> int:
    """vllm_ttkv/layout.py:50-53: each row padded to whole bytes."""
    return (k * bits + 7) // 8


class Geometry:
    """Per-token slot geometry of one layer (vllm_ttkv/layout.py:56-157)."""

    def __init__(self, H, d, r1, qbits, res_k, res_bits, v_lanes, v_bits, align=16):
        self.H, self.d, self.r1, self.qbits = H, d, r1, qbits
        self.res_k, self.res_bits, self.v_lanes, self.v_bits, self.align = (
            res_k, res_bits, v_lanes, v_bits, align)
        self.coeff_bytes = r1 * qbits // 8                                   # :99-105
        self.k_row_bytes = d // 8 + packed_row_bytes(res_k, res_bits) + 2     # :108-110
        self.v_row_bytes = d // 8 + packed_row_bytes(v_lanes, v_bits) + 2     # :112-113
        self.k_slot_bytes = align_up(self.coeff_bytes + 2 + H * self.k_row_bytes, align)  # :138
        self.v_slot_bytes = align_up(H * self.v_row_bytes, align)            # :144
        self.v_offset = self.k_slot_bytes                                    # :122
        self.blob_bytes = self.k_slot_bytes + self.v_slot_bytes              # :151

    def as_dict(self):
        return {k: getattr(self, k) for k in (
            "H", "d", "r1", "qbits", "res_k", "res_bits", "v_lanes", "v_bits", "coeff_bytes",
            "k_row_bytes", "v_row_bytes", "k_slot_bytes", "v_slot_bytes", "v_offset",
            "blob_bytes")}


def geometry_for_config(cfg, r1: int, H: int = 8, d: int = 128) -> Geometry:
    """vllm_ttkv/layout.py:264-275 (`layout_for_config`)."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    return Geometry(H=H, d=d, r1=r1, qbits=cfg["qbits"],
                    res_k=max(int(d * cfg["res_frac"]), 1), res_bits=cfg["res_bits"],
                    v_lanes=cfg["k_lanes"], v_bits=cfg["vbits"])


# ----------------------------------------------------------------------------- bits
def pack_bits_rows(vals: np.ndarray, bits: int) -> np.ndarray:
    """codec/ttkv_packed_cache.py:50-66: [rows, k] codes -> MSB-first stream, row padded to bytes."""
    rows, k = vals.shape
    v = vals.astype(np.int64)
    planes = ((v[:, :, None] >> np.arange(bits - 1, -1, -1)) & 1).astype(np.uint8)
    return np.packbits(planes.reshape(rows, k * bits), axis=1, bitorder="big")


def unpack_bits_rows(packed: np.ndarray, k: int, bits: int) -> np.ndarray:
    """codec/ttkv_packed_cache.py:69-102: inverse of pack_bits_rows -> int32 [rows, k]."""
    rows = packed.shape[0]
    planes = np.unpackbits(packed, axis=1, bitorder="big")[:, :k * bits].reshape(rows, k, bits)
    out = np.zeros((rows, k), np.int32)
    for i in range(bits):                       # plane 0 is the MSB plane
        out = out * 2 + planes[:, :, i].astype(np.int32)
    return out


def pack_mask(mask: np.ndarray) -> np.ndarray:
    """codec/ttkv_packed_cache.py:233-240 (`PackedRows._pack_mask`): lane 8j+b at bit 7-b."""
    return np.packbits(mask.astype(np.uint8), axis=1, bitorder="big")


def unpack_bitmap(bm: np.ndarray, d: int) -> np.ndarray:
    """codec/ttkv_packed_cache.py:138-167 (`unpack_bitmap_rows`)."""
    return np.unpackbits(bm, axis=1, bitorder="big")[:, :d].astype(bool)


# ----------------------------------------------------------------------------- quantisers
def _ruler(x: np.ndarray, divisor: int, ruler_div: str) -> np.ndarray:
    """`x / divisor` with `divisor` a Python int, under torch's CPU ("true") or CUDA ("recip") rule.

    The CUDA rule is a multiply by the fp32 reciprocal (vllm_ttkv/select_triton.py:76-84, :119).
    """
    x = np.asarray(x, np.float32)
    if ruler_div == "recip":
        return (x * (np.float32(1.0) / np.float32(divisor))).astype(np.float32)
    if ruler_div == "true":
        return (x / np.float32(divisor)).astype(np.float32)
    raise ValueError(ruler_div)


def topk_mask(x: np.ndarray, k: int) -> np.ndarray:
    """Exactly k lanes per row by |x| (codec/ttkv_packed_cache.py:179-183, `_topk_mask`).

    torch.topk leaves the tie order unspecified; this picks the lowest lane index among equal
    magnitudes, which is the rule the reference's fused writer fixes (select_triton.py:34-46).
    """
    order = np.argsort(-np.abs(x.astype(np.float32)), axis=1, kind="stable")[:, :k]
    m = np.zeros(x.shape, bool)
    np.put_along_axis(m, order, True, axis=1)
    return m


def packed_rows_build(X: np.ndarray, mask: np.ndarray, k: int, bits: int, ruler_div="recip"):
    """codec/ttkv_packed_cache.py:203-231 (`PackedRows.build`): -> (bitmap, packed, scale fp16)."""
    X = X.astype(np.float32)
    vals = np.where(mask, X, np.float32(0))
    rmax = np.abs(vals).max(axis=1, keepdims=True)
    sc = _ruler(np.where(rmax == 0, np.float32(1), rmax), 2 ** (bits - 1) - 1, ruler_div)
    with np.errstate(invalid="ignore", divide="ignore"):
        q = np.clip(np.rint(vals / sc), -(2 ** (bits - 1)), 2 ** (bits - 1) - 1)
    q = np.where(mask, q, 0) + 2 ** (bits - 1)
    rows = X.shape[0]
    q_rows = q[mask].reshape(rows, k).astype(np.int64)     # row-major order of kept lanes
    return pack_mask(mask), pack_bits_rows(q_rows, bits), sc.reshape(rows).astype(np.float16)


def packed_rows_materialise(bitmap, packed, scale, k: int, bits: int, d: int) -> np.ndarray:
    """codec/ttkv_packed_cache.py:247-271 (`PackedRows.materialise`) in fp32."""
    mask = unpack_bitmap(bitmap, d)
    vals = (unpack_bits_rows(packed, k, bits) - 2 ** (bits - 1)).astype(np.float32)
    vals = vals * scale.astype(np.float32)[:, None]
    out = np.zeros(mask.shape, np.float32)
    out[mask] = vals.reshape(-1)
    return out


def quant_rows(M: np.ndarray, qbits: int, ruler_div="recip"):
    """codec/ttkv_packed_cache.py:170-176 (`_quant_rows`): -> (int8 codes, fp16 ruler)."""
    M = M.astype(np.float32)
    rmax = np.abs(M).max(axis=1, keepdims=True)
    sc = _ruler(np.where(rmax == 0, np.float32(1), rmax), 2 ** (qbits - 1) - 1, ruler_div)
    q = np.clip(np.rint(M / sc), -(2 ** (qbits - 1)), 2 ** (qbits - 1) - 1).astype(np.int8)
    return q, sc.reshape(-1).astype(np.float16)


def quant_coeff(c: np.ndarray, qbits: int, ruler_div="recip"):
    """The per-token coefficient quantiser shared by the fit and the frozen projection
    (codec/ttkv_packed_cache.py:353-356; vllm_ttkv/encode.py:329-333).

    The ruler is taken BEFORE the zero guard here, unlike `_quant_rows`: `amax/127`, then 0 -> 1.
    Returns (codes as float32 in [-128, 127], ruler fp32 [n, 1]).
    """
    c = c.astype(np.float32)
    cs = _ruler(np.abs(c).max(axis=1, keepdims=True), 2 ** (qbits - 1) - 1, ruler_div)
    cs = np.where(cs == 0, np.float32(1), cs).astype(np.float32)
    cq = np.clip(np.rint(c / cs), -(2 ** (qbits - 1)), 2 ** (qbits - 1) - 1).astype(np.float32)
    return cq, cs


# ----------------------------------------------------------------------------- slots
def pack_k_slots(g: Geometry, coeff_q, coeff_scale, bitmap, packed, scale) -> np.ndarray:
    """vllm_ttkv/layout.py:161-193. Residual rows are (head, token) = h*n + i."""
    n = coeff_q.shape[0]
    out = np.zeros((n, g.k_slot_bytes), np.uint8)
    off = 0
    out[:, :g.coeff_bytes] = coeff_q.astype(np.int8).view(np.uint8)
    off = g.coeff_bytes
    out[:, off:off + 2] = coeff_scale.astype(np.float16).view(np.uint8).reshape(n, 2)
    off += 2
    b, p = g.d // 8, packed.shape[1]
    for h in range(g.H):
        rows = slice(h * n, (h + 1) * n)
        out[:, off:off + b] = bitmap[rows]
        off += b
        out[:, off:off + p] = packed[rows]
        off += p
        out[:, off:off + 2] = scale[rows].astype(np.float16).view(np.uint8).reshape(n, 2)
        off += 2
    return out


def unpack_k_slots(g: Geometry, slots: np.ndarray):
    """vllm_ttkv/layout.py:196-219 -> (coeff_q int8, coeff_scale fp16, bitmap, packed, scale)."""
    n = slots.shape[0]
    coeff_q = np.ascontiguousarray(slots[:, :g.coeff_bytes]).view(np.int8)
    off = g.coeff_bytes
    coeff_scale = np.ascontiguousarray(slots[:, off:off + 2]).view(np.float16).reshape(n)
    off += 2
    b, p = g.d // 8, packed_row_bytes(g.res_k, g.res_bits)
    bm = np.empty((g.H * n, b), np.uint8)
    pk = np.empty((g.H * n, p), np.uint8)
    sc = np.empty(g.H * n, np.float16)
    for h in range(g.H):
        rows = slice(h * n, (h + 1) * n)
        bm[rows] = slots[:, off:off + b]
        off += b
        pk[rows] = slots[:, off:off + p]
        off += p
        sc[rows] = np.ascontiguousarray(slots[:, off:off + 2]).view(np.float16).reshape(n)
        off += 2
    return coeff_q, coeff_scale, bm, pk, sc


def pack_v_slots(g: Geometry, bitmap, packed, scale) -> np.ndarray:
    """vllm_ttkv/layout.py:222-239."""
    n = bitmap.shape[0] // g.H
    out = np.zeros((n, g.v_slot_bytes), np.uint8)
    off = 0
    b, p = g.d // 8, packed.shape[1]
    for h in range(g.H):
        rows = slice(h * n, (h + 1) * n)
        out[:, off:off + b] = bitmap[rows]
        off += b
        out[:, off:off + p] = packed[rows]
        off += p
        out[:, off:off + 2] = scale[rows].astype(np.float16).view(np.uint8).reshape(n, 2)
        off += 2
    return out


def unpack_v_slots(g: Geometry, slots: np.ndarray):
    """vllm_ttkv/layout.py:242-261."""
    n = slots.shape[0]
    b, p = g.d // 8, packed_row_bytes(g.v_lanes, g.v_bits)
    bm = np.empty((g.H * n, b), np.uint8)
    pk = np.empty((g.H * n, p), np.uint8)
    sc = np.empty(g.H * n, np.float16)
    off = 0
    for h in range(g.H):
        rows = slice(h * n, (h + 1) * n)
        bm[rows] = slots[:, off:off + b]
        off += b
        pk[rows] = slots[:, off:off + p]
        off += p
        sc[rows] = np.ascontiguousarray(slots[:, off:off + 2]).view(np.float16).reshape(n)
        off += 2
    return bm, pk, sc


# ----------------------------------------------------------------------------- paging, angles
def block_slots(block_row: np.ndarray, seq_len: int, block_size: int) -> np.ndarray:
    """vllm_ttkv/decode.py:307-339: slot id = block_table[r, pos // bs] * bs + pos % bs."""
    pos = np.arange(seq_len)
    return block_row[pos // block_size].astype(np.int64) * block_size + pos % block_size


def cos_sin_from_table(table: np.ndarray, positions: np.ndarray, head_dim: int):
    """vllm_ttkv/decode.py:54-122: vLLM `cat(cos, sin)` table rows -> duplicated fp32 halves."""
    rot = table.shape[-1]
    if rot != head_dim:
        raise NotImplementedError("partial rotary")
    row = table[np.asarray(positions, np.int64)].astype(np.float32)
    c, s = row[:, :rot // 2], row[:, rot // 2:]
    return np.concatenate([c, c], -1), np.concatenate([s, s], -1)


def rope_apply(x, cos, sin):
    """codec/ttkv_packed_cache.py:486-499: x*cos + rotate_half(x)*sin, (j, j+d/2) pairing."""
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return (x * cos + rot * sin).astype(np.float32)


# ----------------------------------------------------------------------------- read
def dense_k(g: Geometry, k_slots: np.ndarray, decoder_f: np.ndarray) -> np.ndarray:
    """vllm_ttkv/reference.py:63-76: raw K [H, n, d] = coefficients @ decoder + residual."""
    n = k_slots.shape[0]
    cq, cs, bm, pk, sc = unpack_k_slots(g, k_slots)
    kflat = (cq.astype(np.float32) * cs.astype(np.float32)[:, None]) @ decoder_f.astype(np.float32)
    R = packed_rows_materialise(bm, pk, sc, g.res_k, g.res_bits, g.d)
    return (kflat.reshape(n, g.H, g.d).transpose(1, 0, 2) + R.reshape(g.H, n, g.d)).astype(np.float32)


def dense_v(g: Geometry, v_slots: np.ndarray) -> np.ndarray:
    """vllm_ttkv/reference.py:79-85: V [H, n, d]."""
    n = v_slots.shape[0]
    bm, pk, sc = unpack_v_slots(g, v_slots)
    return packed_rows_materialise(bm, pk, sc, g.v_lanes, g.v_bits, g.d).reshape(g.H, n, g.d)


def raw_scores(g, k_slots, decoder_f, query, cos, sin, scale=None):
    """vllm_ttkv/reference.py:94-110: scores [n, HQ] with each row rotated by its own position."""
    K_pre = dense_k(g, k_slots, decoder_f)                             # [H, n, d]
    HQ, d = query.shape
    scale = d ** -0.5 if scale is None else scale
    K_post = rope_apply(K_pre.transpose(1, 0, 2), cos[:, None, :], sin[:, None, :])   # [n,H,d]
    p_all = np.arange(HQ) // (HQ // g.H)
    return np.einsum("npd,pd->np", K_post[:, p_all, :], query.astype(np.float32)) * np.float32(scale)


def raw_scores_multi(g, k_slots, decoder_f, query, cos, sin, scale=None, p0=None):
    """vllm_ttkv/reference.py:113-149: scores [HQ, Q, n], causal (row <= p0 + j) when p0 given."""
    K_pre = dense_k(g, k_slots, decoder_f)
    H, n, d = K_pre.shape
    HQ, Q, _ = query.shape
    scale = d ** -0.5 if scale is None else scale
    K_post = rope_apply(K_pre.transpose(1, 0, 2), cos[:, None, :], sin[:, None, :])
    p_all = np.arange(HQ) // (HQ // H)
    s = np.einsum("hqd,phd->hqp", query.astype(np.float32), K_post[:, p_all, :]) * np.float32(scale)
    if p0 is not None:
        pos = p0 + np.arange(Q)
        allow = np.arange(n)[None, :] <= pos[:, None]
        s = np.where(allow[None], s, -np.inf)
    return s.astype(np.float32)


def softmax(x, axis):
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=axis, keepdims=True)


def attend(g, k_slots, v_slots, decoder_f, query, cos, sin, scale=None):
    """vllm_ttkv/reference.py:152-163 (`attend_raw_store`): query [HQ, d] -> [HQ, d]."""
    s = raw_scores(g, k_slots, decoder_f, query, cos, sin, scale)
    p = softmax(s, 0)
    V = dense_v(g, v_slots)
    p_all = np.arange(query.shape[0]) // (query.shape[0] // g.H)
    return np.einsum("np,npd->pd", p, V.transpose(1, 0, 2)[:, p_all, :]).astype(np.float32)


def attend_multi(g, k_slots, v_slots, decoder_f, query, cos, sin, scale=None, p0=None):
    """vllm_ttkv/impl.py:725-778 (`_prefill_continuation`) with the oracle's read: [HQ, Q, d]."""
    s = raw_scores_multi(g, k_slots, decoder_f, query, cos, sin, scale, p0)
    p = softmax(s, -1)
    V = dense_v(g, v_slots)                                            # [H, n, d]
    p_all = np.arange(query.shape[0]) // (query.shape[0] // g.H)
    return np.einsum("hqn,hnd->hqd", p, V[p_all]).astype(np.float32)


def read_blob(cache_u8: np.ndarray, slots: np.ndarray, g: Geometry):
    """vllm_ttkv/decode.py:160-197 + :286-304: gather a request's blobs and split K || V."""
    blob = cache_u8[slots, :g.blob_bytes]
    return blob[:, :g.k_slot_bytes], blob[:, g.k_slot_bytes:g.blob_bytes]


def decode_batch(g, cache_u8, block_table, seq_lens, block_size, queries, decoders, table,
                 scale=None):
    """Decode step over a paged cache: request r attends over its first seq_lens[r] slots.

    queries [B, HQ, d]; decoders: list of [r1, H*d] fp32; table: vLLM cos_sin_cache rows.
    Mirrors vllm_ttkv/impl.py:511-540 per request. Returns [B, HQ, d] fp32.
    """
    out = np.zeros(queries.shape, np.float32)
    for r in range(len(seq_lens)):
        n = int(seq_lens[r])
        slots = block_slots(np.asarray(block_table[r]), n, block_size)
        ks, vs = read_blob(cache_u8, slots, g)
        cos, sin = cos_sin_from_table(table, np.arange(n), g.d)
        out[r] = attend(g, ks, vs, decoders[r], queries[r], cos, sin, scale)
    return out


# ----------------------------------------------------------------------------- write
def tt_svd(X: np.ndarray, tol=0.20, max_rank=None):
    """codec/ttkv_codec.py:78-109: energy-truncated TT-SVD over the given mode order.

    numpy's LAPACK, not torch's: the singular vectors can differ from the reference in sign and
    in the last bits, so a fit run through this is NOT byte-comparable to the reference's. Tests
    pin the fit TAIL by feeding it the reference's own cores instead (`fit_tail`).
    """
    dims = list(X.shape)
    rest = X.reshape(dims[0], -1).astype(np.float32)
    cores, ranks, r_prev = [], [], 1
    for k in range(len(dims) - 1):
        M = rest.reshape(r_prev * dims[k], -1)
        U, S, Vh = np.linalg.svd(M, full_matrices=False)
        U, S, Vh = U.astype(np.float32), S.astype(np.float32), Vh.astype(np.float32)
        e = S ** 2
        tail = np.flip(np.cumsum(np.flip(e))) / (e.sum() + np.float32(1e-30))
        hit = np.nonzero(tail <= np.float32(tol) ** 2)[0]
        r = int(hit[0]) + 1 if hit.size else int(S.size)
        r = max(1, min(r, int(S.size))) if max_rank is None else max(1, min(r, max_rank, int(S.size)))
        ranks.append(r)
        cores.append(U[:, :r].reshape(r_prev, dims[k], r))
        rest = (S[:r, None] * Vh[:r, :]).reshape(r, *dims[k + 1:])
        r_prev = r
    cores.append(rest.reshape(r_prev, dims[-1], 1))
    ranks.append(1)
    return cores, ranks


def quant_cores(cores, qbits, ruler_div="recip"):
    """codec/ttkv_codec.py:142-163 (per-row rulers; the token core is never passed here)."""
    q = 2 ** (qbits - 1) - 1
    out = []
    for c in cores:
        rows = int(c.shape[1]) if int(c.shape[0]) == 1 else int(c.shape[0])   # :124-134
        M = c.reshape(rows, -1).astype(np.float32)
        s = _ruler(np.maximum(np.abs(M).max(axis=1, keepdims=True), np.float32(1e-12)), q, ruler_div)
        out.append((np.clip(np.rint(M / s), -q, q) * s).astype(np.float32).reshape(c.shape))
    return out


def fit_tail(K: np.ndarray, cores, cfg, ruler_div="recip"):
    """Everything in codec/ttkv_packed_cache.py:337-375 (`build_k_layer`) after `tt_svd`.

    K [H, n, d] fp32; cores = (G1 [1,n,r1], G2 [r1,d,r2], G3 [r2,H,1]).
    Returns dict(coeff_q int8 [n,r1], coeff_scale fp16 [n], dec_q int8 [r1,H*d], dec_scale fp16
    [r1], decoder_f fp32, R fp32 [H*n, d], bitmap/packed/scale of the residual).
    """
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    H, n, d = K.shape
    qbits = cfg["qbits"]
    G1, G2, G3 = cores
    r1 = int(G1.shape[2])
    c = G1.reshape(n, r1)
    cq, cs = quant_coeff(c, qbits, ruler_div)
    qc = quant_cores([G2, G3], qbits, ruler_div)
    # dec[a, h, j] = sum_b G2q[a, j, b] * G3q[b, h]   ("ajb,bh->ahj", :361)
    dec = np.einsum("ajb,bh->ahj", qc[0], qc[1][:, :, 0]).astype(np.float32).reshape(r1, H * d)
    dec_q, dec_scale = quant_rows(dec, qbits, ruler_div)
    dec_f = dec_q.astype(np.float32) * dec_scale.astype(np.float32)[:, None]
    kflat = (cq * cs) @ dec_f
    Kd = kflat.reshape(n, H, d).transpose(1, 0, 2)
    R = (K.astype(np.float32) - Kd).reshape(H * n, d).astype(np.float32)
    kr = max(int(d * cfg["res_frac"]), 1)
    mask = topk_mask(R, kr)
    bm, pk, sc = packed_rows_build(R, mask, kr, cfg["res_bits"], ruler_div)
    return dict(coeff_q=cq.astype(np.int8), coeff_scale=cs.reshape(n).astype(np.float16),
                dec_q=dec_q, dec_scale=dec_scale, decoder_f=dec_f.astype(np.float32), R=R,
                bitmap=bm, packed=pk, scale=sc, r1=r1)


def fit_into_budget(K: np.ndarray, g: Geometry, cfg, ruler_div="recip", cores=None):
    """vllm_ttkv/encode.py:257-298: fit capped at the layer's rank budget, zero-padded to it."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    H, n, d = K.shape
    if cores is None:
        cores, _ = tt_svd(np.ascontiguousarray(K.transpose(1, 2, 0)), cfg["tols"], g.r1)
    f = fit_tail(K, cores, cfg, ruler_div)
    r = f["r1"]
    cq = np.zeros((n, g.r1), np.int8)
    cq[:, :r] = f["coeff_q"]
    dec = np.zeros((g.r1, H * d), np.float32)
    dec[:r] = f["decoder_f"]
    f.update(coeff_q=cq, decoder_f=dec, fitted_rank=r)
    return f


def encode_frozen(K: np.ndarray, decoder_f: np.ndarray, pinv: np.ndarray, qbits: int = 8,
                  ruler_div="recip"):
    """vllm_ttkv/encode.py:301-351: project onto a frozen decoder. K [H, n, d].

    Returns (coeff_q int8 [n, r1], coeff_scale fp16 [n], R fp32 [H*n, d]).
    """
    H, n, d = K.shape
    M = K.transpose(1, 0, 2).reshape(n, H * d).astype(np.float32)       # m = h*d + j
    c = (M @ pinv.astype(np.float32)).astype(np.float32)
    cq, cs = quant_coeff(c, qbits, ruler_div)
    kd = ((cq * cs) @ decoder_f.astype(np.float32)).reshape(n, H, d).transpose(1, 0, 2)
    R = (K.astype(np.float32) - kd).reshape(H * n, d).astype(np.float32)
    return cq.astype(np.int8), cs.reshape(n).astype(np.float16), R


def encode_rows(X: np.ndarray, lanes: int, bits: int, ruler_div="recip"):
    """Top-k select + PackedRows.build over (head, token) rows: the residual and V write
    (codec/ttkv_packed_cache.py:371-385; vllm_ttkv/select_triton.py:157-232)."""
    mask = topk_mask(X, lanes)
    return packed_rows_build(X, mask, lanes, bits, ruler_div)


def build_slots(g: Geometry, coeff_q, coeff_scale, R, V, ruler_div="recip"):
    """Token blobs [n, blob] for one request's store: coefficient block, K residual, V rows.
    R [H*n, d] (head, token); V [H, n, d]. vllm_ttkv/encode.py:582-603 (torch branch)."""
    bm, pk, sc = encode_rows(R, g.res_k, g.res_bits, ruler_div)
    ks = pack_k_slots(g, coeff_q, coeff_scale, bm, pk, sc)
    H, n, d = V.shape
    vbm, vpk, vsc = encode_rows(V.reshape(H * n, d).astype(np.float32), g.v_lanes, g.v_bits,
                                ruler_div)
    vs = pack_v_slots(g, vbm, vpk, vsc)
    return np.concatenate([ks, vs], axis=1)
