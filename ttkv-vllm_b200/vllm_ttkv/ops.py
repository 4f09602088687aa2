"""torch-facing wrappers of the C ABI: device tensors in, launches on torch's current stream.

Every function validates shapes and dtypes on the host, hands raw pointers to
`libttkv_sm100.so`, and never reads a device value back. Device-side refusals (a block index
outside the cache, a PAD_SLOT_ID slot, a decoder index outside the pool) land in a per-device
status word; `check_status()` reads it once (one readback) and raises.
"""
from __future__ import annotations

import ctypes as C

import torch

from vllm_ttkv import _lib
from vllm_ttkv.layout import TTKLayout

_DTYPE = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}

_STATUS: dict = {}
_PINNED: dict = {}                       # data_ptr -> tensor a captured graph reads
_WORKSPACE: dict = {}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE[t.dtype]
    except KeyError:
        raise TypeError(f"dtype {t.dtype} is not one of float32/float16/bfloat16") from None


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError(f"expected a CUDA tensor, got one on {t.device}: the TT-KV ops run "
                             f"only on the GPU (no CPU path)")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def capturing() -> bool:
    """Whether the current stream is capturing a CUDA graph."""
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


def pin(*tensors: torch.Tensor) -> None:
    """Keep `tensors` alive for the rest of the process: a captured CUDA graph holds their raw
    addresses (passed through the C ABI), which torch does not know about."""
    for t in tensors:
        _PINNED[t.data_ptr()] = t


def is_pinned(t: torch.Tensor) -> bool:
    return _PINNED.get(t.data_ptr()) is t


def status_word(device=None) -> torch.Tensor:
    """The per-device int32 status the kernels report device-side refusals into."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    t = _STATUS.get(dev)
    if t is None:
        if capturing():
            raise RuntimeError("the status word must exist before a CUDA graph capture (its zero "
                               "fill would rerun at every replay): run one eager step first")
        t = torch.zeros(1, dtype=torch.int32, device=dev)
        _STATUS[dev] = t
    return t


def reset_status(device=None) -> None:
    status_word(device).zero_()


def check_status(device=None) -> None:
    """Read the status word (a device readback) and raise if a kernel recorded a refusal."""
    code = int(status_word(device).item())
    if code:
        reset_status(device)
        msg = _lib.STATUS.get(code, f"code {code}")
        if code in (1, 4):
            raise IndexError(f"vllm_ttkv: {msg}")
        raise RuntimeError(f"vllm_ttkv: {msg}")


def workspace(nbytes: int, device, key="read") -> torch.Tensor:
    """A cached byte buffer of at least `nbytes` (grown, never shrunk) for kernel scratch."""
    dev = torch.device(device)
    buf = _WORKSPACE.get((dev, key))
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8, device=dev)
        _WORKSPACE[(dev, key)] = buf
    if capturing():                        # a graph keeps the scratch it launched with
        pin(buf)
    return buf


def byte_view(cache: torch.Tensor) -> torch.Tensor:
    """`[n_slots, row_bytes]` uint8 view of a layer's page `[blocks, (1,) block_size, C]` in any
    dtype (vLLM allocates it in the model dtype with C counted in elements,
    vllm_ttkv/decode.py:125-157)."""
    c = cache
    if c.dim() == 4:
        if c.shape[1] != 1:
            raise ValueError(f"expected num_head_slots=1, got a cache of shape {tuple(c.shape)}")
        c = c[:, 0]
    if c.dim() != 3:
        raise ValueError(f"expected a [num_blocks, block_size, C] page, got {tuple(cache.shape)}")
    try:
        u8 = c if c.dtype == torch.uint8 else c.view(torch.uint8)
    except RuntimeError as e:
        raise RuntimeError(f"the cache page {tuple(cache.shape)} {cache.dtype} cannot be viewed as "
                           f"bytes ({e})") from e
    if not u8.is_contiguous():
        raise ValueError("the cache page must be contiguous")
    return u8.reshape(-1, u8.shape[-1])


def _row_stride(t: torch.Tensor, name: str) -> int:
    """Stride between tokens of a [n, heads, 128] tensor whose [heads, 128] rows are contiguous.
    Size-1 dimensions may carry any stride (numpy views and broadcasts produce those)."""
    if t.dim() != 3 or t.shape[2] != 128:
        raise ValueError(f"{name} must be [n, heads, 128], got {tuple(t.shape)}")
    if (t.shape[2] > 1 and t.stride(2) != 1) or (t.shape[1] > 1 and t.stride(1) != 128):
        raise ValueError(f"{name} must have contiguous [heads, 128] rows (strides {t.stride()})")
    return t.stride(0) if t.shape[0] > 1 else t.shape[1] * 128


def _cache_struct(lay: TTKLayout, flat: torch.Tensor, block_size: int, flags: int = 0) -> _lib.Cache:
    if flat.dtype != torch.uint8 or flat.dim() != 2:
        raise ValueError("cache must be a [n_slots, row_bytes] uint8 view")
    if flat.shape[1] < lay.compressed_bytes_per_token():
        raise ValueError(f"cache rows are {flat.shape[1]} bytes, the layout needs "
                         f"{lay.compressed_bytes_per_token()}")
    return _lib.Cache(flat.data_ptr(), flat.shape[0], flat.stride(0), block_size, flags)


def _lead_stride(t: torch.Tensor) -> int:
    """Elements between consecutive rows of a contiguous pool. A size-1 leading dimension may carry
    any stride (a numpy `x[None]` view has 0), so it is derived from the other dimensions."""
    if t.shape[0] > 1:
        return t.stride(0)
    n = 1
    for d in t.shape[1:]:
        n *= d
    return n


def decoder_image(lay: TTKLayout, decoders: torch.Tensor, out=None):
    """The decode's operand images of decoders [n, r1, H*d] fp32: (image [n, bytes] uint8,
    scales [n, H] fp32), or None when the tensor-core decode does not serve the layout.
    `out` (image, scales) are written in place when given."""
    _need_cuda(decoders)
    if decoders.dtype != torch.float32 or decoders.dim() != 3 or not decoders.is_contiguous():
        raise TypeError("decoders must be a contiguous float32 [n, r1, H*d] pool")
    L = _lib.lib()
    la = lay.abi()
    per = L.ttkv_decoder_image_bytes(C.byref(la))
    if per == 0:
        return None
    n = decoders.shape[0]
    if out is None:
        image = torch.zeros(n, per, dtype=torch.uint8, device=decoders.device)
        scales = torch.zeros(n, lay.H, dtype=torch.float32, device=decoders.device)
    else:
        image, scales = out
        if image.dtype != torch.uint8 or image.shape[0] < n or image.stride(0) < per or scales.shape[0] < n:
            raise ValueError("image / scales too small for the decoders")
    _lib.check(L.ttkv_decoder_image(C.byref(la), decoders.data_ptr(), _lead_stride(decoders), n,
                                    image.data_ptr(), image.stride(0), scales.data_ptr(), _stream()))
    return image, scales


def _batch_struct(block_table, seq_lens, decoders, dec_index, images=None) -> _lib.Batch:
    for name, t, dt in (("block_table", block_table, torch.int32), ("seq_lens", seq_lens, torch.int32),
                        ("dec_index", dec_index, torch.int32), ("decoders", decoders, torch.float32)):
        if t.dtype != dt:
            raise TypeError(f"{name} must be {dt}, got {t.dtype}")
    if block_table.dim() != 2 or block_table.stride(1) != 1:
        raise ValueError("block_table must be [n_reqs, max_blocks] with unit column stride")
    if decoders.dim() != 3 or not decoders.is_contiguous():
        raise ValueError("decoders must be a contiguous [n_decoders, r1, H*d] float32 pool")
    n = block_table.shape[0]
    if seq_lens.numel() < n or dec_index.numel() < n:
        raise ValueError("seq_lens / dec_index shorter than the block table")
    img, istride, scl = None, 0, None
    if images is not None:
        image, scales = images
        if image.shape[0] < decoders.shape[0] or scales.shape[0] < decoders.shape[0]:
            raise ValueError("one decoder image and scale row per pool row")
        img, istride, scl = image.data_ptr(), image.stride(0), scales.data_ptr()
    return _lib.Batch(block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
                      seq_lens.data_ptr(), n, decoders.data_ptr(), _lead_stride(decoders),
                      dec_index.data_ptr(), decoders.shape[0], img, istride, scl)


def _rope_struct(table: torch.Tensor) -> _lib.Rope:
    if table.dim() != 2 or table.shape[1] != 128 or not table.is_contiguous():
        raise ValueError(f"the RoPE table must be a contiguous [max_pos, 128] cos||sin table, got "
                         f"{tuple(table.shape)} (partial rotary is refused, vllm_ttkv/decode.py:92)")
    return _lib.Rope(table.data_ptr(), dtype_code(table), table.shape[0])


def decode_paged(lay: TTKLayout, cache: torch.Tensor, block_size: int, block_table: torch.Tensor,
                 seq_lens: torch.Tensor, decoders: torch.Tensor, dec_index: torch.Tensor,
                 table: torch.Tensor, q: torch.Tensor, scale: float, out: torch.Tensor,
                 max_seq_len: int, head_lo: int = 0, head_hi: int | None = None,
                 status: torch.Tensor | None = None, images=None, peers=None) -> torch.Tensor:
    """Batched decode read: q [B, HQ, d] (row r = request r) -> out [B, HQ, d] (heads of the KV
    heads [head_lo, head_hi) written). `cache` is the [n_slots, row_bytes] uint8 view. `images`:
    the pool's (image, scales) from `decoder_image`, staged instead of converting the decoders.
    `peers` (a `_lib.Peers` for this layer, see `shard.PeerGather`): the merge also stores the rows
    into every other rank's `out` and counts its arrivals there (`ttkv_decode_paged_gather`); the
    caller then waits with `peer_wait` before reading the other ranks' heads."""
    _need_cuda(cache, block_table, seq_lens, decoders, dec_index, table, q, out)
    head_hi = lay.H if head_hi is None else head_hi
    B, HQ, d = q.shape
    qs, os_ = _row_stride(q, "q"), _row_stride(out, "out")
    if out.shape[0] < B or block_table.shape[0] != B:
        raise ValueError(f"{B} queries, {block_table.shape[0]} block-table rows, {out.shape[0]} outputs")
    L = _lib.lib()
    la = lay.abi()
    ws_n = L.ttkv_decode_workspace_bytes(C.byref(la), B, HQ, max_seq_len, head_lo, head_hi)
    ws = workspace(ws_n, q.device)
    st = status if status is not None else status_word(q.device)
    c_s = _cache_struct(lay, cache, block_size)
    b_s = _batch_struct(block_table, seq_lens, decoders, dec_index, images)
    r_s = _rope_struct(table)
    if peers is None:
        _lib.check(L.ttkv_decode_paged(
            C.byref(la), C.byref(c_s), C.byref(b_s), C.byref(r_s), q.data_ptr(), dtype_code(q),
            qs, HQ, float(scale), head_lo, head_hi, out.data_ptr(), dtype_code(out),
            os_, int(max_seq_len), ws.data_ptr(), ws.numel(), st.data_ptr(), _stream()))
    else:
        _lib.check(L.ttkv_decode_paged_gather(
            C.byref(la), C.byref(c_s), C.byref(b_s), C.byref(r_s), q.data_ptr(), dtype_code(q),
            qs, HQ, float(scale), head_lo, head_hi, out.data_ptr(), dtype_code(out),
            os_, int(max_seq_len), ws.data_ptr(), ws.numel(), C.byref(peers), st.data_ptr(), _stream()))
    return out


def peer_wait(peers, arrivals: int, status: torch.Tensor | None = None) -> None:
    """Wait on the device (stream-ordered, bounded) until every rank's merge of this step has
    stored its rows into this rank's output (`ttkv_peer_wait`); `arrivals` = world * G * KV heads
    per rank * requests of the step."""
    st = status if status is not None else status_word()
    _lib.check(_lib.lib().ttkv_peer_wait(C.byref(peers), int(arrivals), st.data_ptr(), _stream()))


def prefill_cont_paged(lay: TTKLayout, cache: torch.Tensor, block_size: int,
                       block_table: torch.Tensor, seq_lens: torch.Tensor, decoders: torch.Tensor,
                       dec_index: torch.Tensor, table: torch.Tensor, q_start: torch.Tensor,
                       q_len: torch.Tensor, q: torch.Tensor, scale: float, out: torch.Tensor,
                       max_q_len: int, max_seq_len: int, head_lo: int = 0,
                       head_hi: int | None = None, status: torch.Tensor | None = None, images=None):
    """Continuation read: request r's queries are rows q_start[r] .. +q_len[r] of q [N, HQ, d],
    at positions seq_len - q_len + j, causal over the stored rows. `images`: the pool's
    (image, scales) from `decoder_image`, staged by the tensor-core path instead of converting."""
    _need_cuda(cache, block_table, seq_lens, decoders, dec_index, table, q_start, q_len, q, out)
    head_hi = lay.H if head_hi is None else head_hi
    N, HQ, d = q.shape
    qs, os_ = _row_stride(q, "q"), _row_stride(out, "out")
    for name, t in (("q_start", q_start), ("q_len", q_len)):
        if t.dtype != torch.int32:
            raise TypeError(f"{name} must be int32")
    L = _lib.lib()
    la = lay.abi()
    B = block_table.shape[0]
    st = status if status is not None else status_word(q.device)
    c_s = _cache_struct(lay, cache, block_size)
    b_s = _batch_struct(block_table, seq_lens, decoders, dec_index, images)
    r_s = _rope_struct(table)

    def call(ws_ptr, ws_n):
        return L.ttkv_prefill_cont_paged(
            C.byref(la), C.byref(c_s), C.byref(b_s), C.byref(r_s), q_start.data_ptr(), q_len.data_ptr(),
            q.data_ptr(), dtype_code(q), qs, HQ, float(scale), head_lo, head_hi,
            out.data_ptr(), dtype_code(out), os_, int(max_q_len), int(max_seq_len),
            ws_ptr, ws_n, st.data_ptr(), _stream())

    # the tensor-core continuation (decoder images given) needs no workspace: call without one
    # first; a path that needs one answers TTKV_ERR_WORKSPACE before it launches anything, and
    # only then is the workspace sized (hundreds of MB at 256-query chunks) and the call repeated
    code = call(None, 0) if images is not None else _lib.ERR_WORKSPACE
    if code == _lib.ERR_WORKSPACE:
        ws_n = L.ttkv_prefill_workspace_bytes(C.byref(la), B, HQ, max_q_len, max_seq_len, head_lo, head_hi)
        ws = workspace(ws_n, q.device)
        code = call(ws.data_ptr(), ws.numel())
    _lib.check(code)
    return out


def write_paged(lay: TTKLayout, cache: torch.Tensor, slot_mapping: torch.Tensor, k: torch.Tensor,
                v: torch.Tensor, tok_dec: torch.Tensor, decoders: torch.Tensor,
                pinvs: torch.Tensor | None = None, coeff_q: torch.Tensor | None = None,
                coeff_scale: torch.Tensor | None = None, status: torch.Tensor | None = None,
                skip_pad: bool = False, heads: tuple[int, int] | None = None):
    """Encode tokens k/v [n, H, d] (raw pre-RoPE K; V) into their slots.

    Frozen path: `pinvs` [n_dec, r1, H*d] (pinv transposed) given -> project + quantise.
    Fit path: `coeff_q` [n, r1] int8 and `coeff_scale` [n] float32 given.
    skip_pad: a negative slot (PAD_SLOT_ID, the padding of a batch padded to a captured graph's
    size) is skipped instead of refused.
    heads: (h_lo, h_hi) for a storage-sharded cache holding only those KV heads (rows of
    `lay.shard(h_lo, h_hi)`); k, v, the decoders and pinvs still cover every head of `lay`."""
    _need_cuda(cache, slot_mapping, k, v, tok_dec, decoders)
    n = slot_mapping.numel()
    if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous():
        raise TypeError("slot_mapping must be contiguous int64")
    for name, t in (("k", k), ("v", v)):
        if t.dim() != 3 or t.shape[1:] != (lay.H, lay.d):
            raise ValueError(f"{name} must be [n, {lay.H}, {lay.d}], got {tuple(t.shape)}")
        _row_stride(t, name)
        if t.shape[0] < n:
            raise ValueError(f"{name} holds {t.shape[0]} tokens for {n} slot ids")
    if tok_dec.dtype != torch.int32 or tok_dec.numel() < n:
        raise TypeError("tok_dec must be int32 with one entry per token")
    if decoders.dtype != torch.float32 or decoders.dim() != 3 or not decoders.is_contiguous():
        raise TypeError("decoders must be a contiguous float32 [n_dec, r1, H*d] pool")
    L = _lib.lib()
    la = lay.abi()
    st = status if status is not None else status_word(k.device)
    h_lo, h_hi = (0, lay.H) if heads is None else (int(heads[0]), int(heads[1]))
    c_s = _cache_struct(lay.shard(h_lo, h_hi), cache, 1, _lib.CACHE_SKIP_PAD if skip_pad else 0)
    ws_n = L.ttkv_write_workspace_bytes(C.byref(la), n)
    ws = workspace(ws_n, k.device, key="write")
    if pinvs is not None:
        if pinvs.shape != decoders.shape or not pinvs.is_contiguous() or pinvs.dtype != torch.float32:
            raise ValueError("pinvs must match the decoder pool's shape, contiguous float32")
        pv, pv_stride, cq, cs = pinvs.data_ptr(), _lead_stride(pinvs), None, None
    else:
        if coeff_q is None or coeff_scale is None:
            raise ValueError("the fit path needs coeff_q and coeff_scale")
        if coeff_q.dtype != torch.int8 or coeff_q.shape != (n, lay.r1) or not coeff_q.is_contiguous():
            raise ValueError(f"coeff_q must be contiguous int8 [{n}, {lay.r1}]")
        if coeff_scale.dtype != torch.float32 or coeff_scale.numel() != n:
            raise ValueError("coeff_scale must be float32 [n]")
        pv, pv_stride, cq, cs = None, 0, coeff_q.data_ptr(), coeff_scale.contiguous().data_ptr()
    _lib.check(L.ttkv_write_paged_shard(
        C.byref(la), h_lo, h_hi, C.byref(c_s), slot_mapping.data_ptr(), n, k.data_ptr(), dtype_code(k),
        _row_stride(k, "k"), v.data_ptr(), dtype_code(v), _row_stride(v, "v"), tok_dec.data_ptr(),
        decoders.data_ptr(), _lead_stride(decoders), pv, pv_stride, decoders.shape[0], cq, cs,
        ws.data_ptr(), ws.numel(), st.data_ptr(), _stream()))


def select_pack_rows(cache: torch.Tensor, slots: torch.Tensor, x: torch.Tensor, *, field_off: int,
                     row_stride: int, lanes: int, bits: int, heads: int, d: int,
                     status: torch.Tensor | None = None):
    """`select_triton.write_rows`' contract: x [heads*n_tok, d] in (head, token) order."""
    _need_cuda(cache, slots, x)
    if x.dim() != 2 or x.shape[1] != d or not x.is_contiguous():
        raise ValueError(f"x must be a contiguous [rows, {d}] tensor")
    n_tok = slots.numel()
    if x.shape[0] != n_tok * heads:
        raise ValueError(f"{x.shape[0]} rows for {n_tok} tokens and {heads} heads")
    sl = slots.to(torch.int64).contiguous()
    st = status if status is not None else status_word(x.device)
    c_s = _lib.Cache(cache.data_ptr(), cache.shape[0], cache.stride(0), 1, 0)
    _lib.check(_lib.lib().ttkv_select_pack_rows(
        C.byref(c_s), sl.data_ptr(), n_tok, x.data_ptr(), dtype_code(x), heads, d, field_off,
        row_stride, lanes, bits, st.data_ptr(), _stream()))


def fit_tail(G1, G2, G3, budget: int, qbits: int = 8):
    """Everything build_k_layer does after the SVDs, on the device.

    G1 [n, r], G2 [r, d, r2], G3 [r2, H] float32 -> dict(coeff_q int8 [n, budget], coeff_scale
    float32 [n], dec_q int8 [r, H*d], dec_scale float16 [r], decoder float32 [budget, H*d])."""
    _need_cuda(G1, G2, G3)
    G1, G2, G3 = (t.float().contiguous() for t in (G1, G2, G3))
    n, r = G1.shape
    r_, d, r2 = G2.shape
    H = G3.shape[1]
    if r_ != r or G3.shape[0] != r2:
        raise ValueError("core shapes disagree")
    dev = G1.device
    out = dict(coeff_q=torch.empty(n, budget, dtype=torch.int8, device=dev),
               coeff_scale=torch.empty(n, dtype=torch.float32, device=dev),
               dec_q=torch.empty(r, H * d, dtype=torch.int8, device=dev),
               dec_scale=torch.empty(r, dtype=torch.float16, device=dev),
               decoder=torch.empty(budget, H * d, dtype=torch.float32, device=dev))
    L = _lib.lib()
    nb = L.ttkv_fit_tail_scratch_bytes(r, r2, H, d)
    scratch = workspace(nb, dev, key="fit")
    _lib.check(L.ttkv_fit_tail(
        G1.data_ptr(), G2.data_ptr(), G3.data_ptr(), n, r, r2, H, d, qbits, budget,
        out["coeff_q"].data_ptr(), out["coeff_scale"].data_ptr(), out["dec_q"].data_ptr(),
        out["dec_scale"].data_ptr(), out["decoder"].data_ptr(), scratch.data_ptr(), scratch.numel(),
        _stream()))
    return out
