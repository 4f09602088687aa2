"""Device memory a TT-KV deployment needs besides its cache, for an engine's profiling pass.

An engine that sizes its KV cache from the memory left after profiling (vLLM does) has to see
everything else the backend will hold, or the 4.5x smaller format does not become 4.5x more cached
tokens: memory taken after the profile can push a later allocation out of memory. No counterpart
in the reference (its transient buffers are allocated per call, README.md:640-653).

Three parts, all from the library's own sizing functions (host code, no GPU needed):
* `step_scratch_bytes`: the largest scratch one step asks for (decode, continuation, write),
  which the ops keep cached and reuse (`ops.workspace`);
* `decoder_pool_bytes`: the decoder pools per live request (decoders, pseudo-inverses and the
  decode's operand images, every layer);
* `cache_bytes_per_token`: the packed slot bytes per cached token over the layers, to turn the
  remaining memory into a token capacity (`tokens_that_fit`).
"""
from __future__ import annotations

import ctypes as C

from vllm_ttkv import _lib


TC_CONTINUATION_MAX_R1 = 126     # the tensor-core continuation's largest rank (no scratch)


def tc_continuation_serves(lay, HQ: int) -> bool:
    """Whether a continuation of this layout can take the tensor-core continuation (which needs no
    scratch) when it is called with the decoders' images and a 16-bit query: the layout fields the
    library checks (ttkv_read.cu, `tc_serves` and `ct_serves`): d = 128, 8-bit coefficients whose
    block with its 2-byte scale fits one 128-byte row, codes of at most 4 bits over at most 128
    lanes, a GQA group of at most 8. Where the library still refuses a call (its alignment checks),
    `ops.prefill_cont_paged` retries it with the 8-row plan's workspace."""
    G = HQ // lay.H if lay.H and HQ % lay.H == 0 else 0
    return (lay.d == 128 and lay.qbits == 8 and 1 <= G <= 8 and lay.r1 <= TC_CONTINUATION_MAX_R1 and
            lay.coeff_bytes + 2 <= 128 and lay.res_bits <= 4 and lay.v_bits <= 4 and
            lay.res_k <= 128 and lay.v_lanes <= 128)


def step_scratch_bytes(layouts, max_reqs: int, max_q_len: int, max_seq_len: int, HQ: int,
                       max_tokens: int | None = None, tc_continuation: bool = False) -> int:
    """The largest scratch a step takes over the layers: a decode of `max_reqs` requests, a
    continuation of `max_reqs` chunks of up to `max_q_len` queries, a frozen write of `max_tokens`
    tokens (default max_reqs * max_q_len), each bounded by `max_seq_len`, and a fit's tail. The
    read, write and fit scratch are separate cached buffers, so the result is their sum. A first
    chunk's two decompositions (torch) take temporaries of their own (the [n, H*d] fp32 unfolding
    and its copies, a few times 4 * n * H*d bytes for n tokens), which a profiling run that
    includes a prefill of that length sees.

    tc_continuation: the continuations run with the decoder pools' images and 16-bit queries (as
    `TTKVAttentionImpl` calls them), so a layer that `tc_continuation_serves` takes the tensor-core
    continuation, which needs no scratch; by default every layer is counted with the 8-row plan's
    workspace, the bound for any call."""
    L = _lib.lib()
    max_tokens = max_reqs * max_q_len if max_tokens is None else max_tokens
    read = cont = write = fit = 0
    for lay in layouts:
        fit = max(fit, L.ttkv_fit_tail_scratch_bytes(lay.r1, lay.H, lay.H, lay.d))
        la = lay.abi()
        read = max(read, L.ttkv_decode_workspace_bytes(C.byref(la), max_reqs, HQ, max_seq_len, 0, lay.H))
        if max_q_len > 1 and not (tc_continuation and tc_continuation_serves(lay, HQ)):
            cont = max(cont, L.ttkv_prefill_workspace_bytes(C.byref(la), max_reqs, HQ, max_q_len,
                                                            max_seq_len, 0, lay.H))
        write = max(write, L.ttkv_write_workspace_bytes(C.byref(la), max_tokens))
    # the continuation shares the decode's cached buffer (ops.workspace key "read")
    return max(read, cont) + write + fit


def decoder_pool_bytes(layouts, n_requests: int) -> int:
    """Decoder-pool memory of `n_requests` live requests over the layers: per layer and request a
    decoder and a transposed pseudo-inverse ([r1, H*d] fp32 each), the decode's operand image and
    its H scales."""
    L = _lib.lib()
    per = 0
    for lay in layouts:
        per += 2 * lay.r1 * lay.H * lay.d * 4
        per += int(L.ttkv_decoder_image_bytes(C.byref(lay.abi()))) + lay.H * 4
    return per * n_requests


def cache_bytes_per_token(layouts) -> int:
    """Packed slot bytes of one cached token over the layers (25,328 B for the 28 calibrated
    Llama-3.2-3B layers at `safe`)."""
    return sum(lay.compressed_bytes_per_token() for lay in layouts)


def tokens_that_fit(layouts, free_bytes: int, max_reqs: int, max_q_len: int, max_seq_len: int,
                    HQ: int, tc_continuation: bool = False) -> int:
    """Cached tokens that fit in `free_bytes` once a step's scratch and the decoder pools of
    `max_reqs` requests are set aside (`tc_continuation` as for `step_scratch_bytes`)."""
    rest = free_bytes - step_scratch_bytes(layouts, max_reqs, max_q_len, max_seq_len, HQ,
                                           tc_continuation=tc_continuation) \
        - decoder_pool_bytes(layouts, max_reqs)
    return max(0, rest // cache_bytes_per_token(layouts))

