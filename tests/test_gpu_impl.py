"""The vLLM-facing adapter end to end on the GPU: `TTKVAttentionImpl.forward` writes the step's
tokens and reads attention, checked against the CPU oracle evaluated on the cache bytes after the
write (the reference's tests/test_impl_decode.py cases: batched decode, continuation, first chunk,
a mixed batch, two layers of one step)."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import stores
from oracle import ttkv_oracle as O
from vllm_ttkv import encode, metadata, patch, rope_store
from vllm_ttkv import synthetic as S
from vllm_ttkv.impl import TTKVAttentionImpl
from vllm_ttkv.layout import TTKLayout

pytestmark = pytest.mark.gpu

HQ, H, D = 24, 8, 128
SCALE = D ** -0.5
ATOL = 2e-3                      # read-path tolerance on attention outputs (fp16 store)


@pytest.fixture(autouse=True)
def _clean():
    rope_store.clear_decoders()
    rope_store.clear_stores()
    patch.clear_stash()
    yield
    rope_store.clear_decoders()
    rope_store.clear_stores()
    patch.clear_stash()


def _lay(g):
    return TTKLayout(H=g.H, d=g.d, r1=g.r1, qbits=g.qbits, res_k=g.res_k, res_bits=g.res_bits,
                     v_lanes=g.v_lanes, v_bits=g.v_bits)


def _world(seed, seq_lens, fresh=(), cfg="safe", r1=32, name="model.layers.0.self_attn.attn"):
    """An oracle-built store on the GPU; requests not in `fresh` get their decoders registered."""
    st = stores.make_store(seed, seq_lens, cfg=cfg, r1=r1)
    g = st["g"]
    lay = _lay(g)
    bs = st["block_size"]
    page = torch.from_numpy(st["cache"]).cuda().reshape(-1, 1, bs, g.blob_bytes)
    table = torch.from_numpy(st["table"]).cuda().half()
    layer = SimpleNamespace(layer_name=name, ttkv_layout=lay,
                            rotary_emb=SimpleNamespace(cos_sin_cache=table))
    for r in range(len(seq_lens)):
        if r not in fresh:
            dec = encode.KDecoder(torch.from_numpy(st["decoders"][r]).cuda())
            rope_store.register_decoder(name, int(st["block_table"][r][0]), dec, lay=lay)
    return dict(st=st, g=g, lay=lay, page=page, table=table, layer=layer, bs=bs)


def _step(w, q_lens, seed=0):
    """This step's tokens (the last q_lens[r] positions of each request): metadata and inputs."""
    st, bs = w["st"], w["bs"]
    slots, ks, vs = [], [], []
    for r, ql in enumerate(q_lens):
        n = int(st["seq_lens"][r])
        pos = np.arange(n - ql, n)
        slots.append(O.block_slots(st["block_table"][r], n, bs)[pos])
        K, V = st["kv"][r]
        ks.append(K[:, pos].transpose(1, 0, 2))
        vs.append(V[:, pos].transpose(1, 0, 2))
    N = sum(q_lens)
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32)
    md = metadata.TTKVAttentionMetadata(
        seq_lens=torch.from_numpy(st["seq_lens"]).cuda(),
        slot_mapping=torch.from_numpy(np.concatenate(slots).astype(np.int64)).cuda(),
        block_table=torch.from_numpy(st["block_table"]).cuda(),
        query_start_loc=qsl.cuda(), query_start_loc_cpu=qsl, num_actual_tokens=N,
        ttkv_serial=metadata.next_serial())
    raw_k = torch.from_numpy(np.concatenate(ks)).cuda().half()
    value = torch.from_numpy(np.concatenate(vs)).cuda().half()
    q = torch.from_numpy(S.synth_queries(seed + 7, (N, HQ, D), "float16")).cuda().half()
    return md, raw_k, value, q


def _forward(impl, w, md, raw_k, value, q, key=None):
    patch.stash_raw_k(w["layer"].layer_name, raw_k, None, w["table"])
    out = torch.full((q.shape[0], HQ, D), float("nan"), dtype=torch.float16, device="cuda")
    impl.forward(w["layer"], q, key, value, w["page"], md, out)
    torch.cuda.synchronize()
    return out


def _after(w):
    """The oracle's view of the store after the step's write."""
    st = dict(w["st"])
    st["cache"] = w["page"].reshape(-1, w["g"].blob_bytes).cpu().numpy()
    return st


def _close(got, want):
    want16 = want.astype(np.float16).astype(np.float32)
    err = np.abs(got.float().cpu().numpy() - want16).max()
    assert err < ATOL, err


def test_batched_decode_writes_each_token_then_reads_every_request():
    w = _world(31, [70, 33, 129, 17])
    md, raw_k, value, q = _step(w, [1, 1, 1, 1])
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    out = _forward(impl, w, md, raw_k, value, q)
    st = _after(w)
    _close(out, stores.expected_decode(st, q=q.float().cpu().numpy()))
    # the written rows are the oracle's frozen encoding of the step's raw keys
    g = w["g"]
    for r in range(4):
        n = int(st["seq_lens"][r])
        slot = O.block_slots(st["block_table"][r], n, w["bs"])[n - 1]
        # the impl receives the model's fp16 K and V, so the oracle encodes the same values
        K, V = (x[:, n - 1:n].astype(np.float16).astype(np.float32) for x in st["kv"][r])
        cq, cs, R = O.encode_frozen(K, st["decoders"][r], st["pinvT"][r].T)
        want = O.build_slots(g, cq, cs, R, V)[0]
        got = st["cache"][slot]
        assert np.array_equal(got[g.v_offset:], want[g.v_offset:])
        assert (got == want).mean() > 0.99


def test_continuation_chunk_reads_the_whole_store_causally():
    w = _world(32, [70, 45])
    md, raw_k, value, q = _step(w, [6, 9])
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    out = _forward(impl, w, md, raw_k, value, q)
    st = _after(w)
    qn = q.float().cpu().numpy()
    _close(out[:6], stores.expected_continuation(st, 0, qn[:6].transpose(1, 0, 2)).transpose(1, 0, 2))
    _close(out[6:], stores.expected_continuation(st, 1, qn[6:].transpose(1, 0, 2)).transpose(1, 0, 2))


def test_first_chunk_attends_over_its_own_keys_fits_a_decoder_and_the_next_step_decodes_it():
    n = 40
    w = _world(33, [n + 1], fresh=(0,))
    st = w["st"]
    # step 1: the first chunk (positions 0..n-1), seq_len == q_len
    md, raw_k, value, q = _step(dict(w, st=dict(st, seq_lens=np.array([n], np.int32))), [n])
    key = torch.randn(n, H, D, device="cuda").half()           # the model's post-RoPE key
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    out = _forward(impl, w, md, raw_k, value, q, key=key)
    G = HQ // H
    qf = q.float().transpose(0, 1)[None]
    kf = key.float().repeat_interleave(G, 1).transpose(0, 1)[None]
    vf = value.float().repeat_interleave(G, 1).transpose(0, 1)[None]
    ref = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=True, scale=SCALE)
    assert (out.float() - ref[0].transpose(0, 1)).abs().max().item() < 2e-2
    kdec = rope_store.decoder_for_request(w["layer"].layer_name, int(st["block_table"][0][0]))
    assert kdec is not None
    # step 2: one decode token at position n, projected onto the fitted decoder and read back
    md2, raw_k2, value2, q2 = _step(w, [1], seed=1)
    out2 = _forward(impl, w, md2, raw_k2, value2, q2)
    st2 = _after(w)
    st2["decoders"] = kdec.decoder_f.cpu().numpy()[None]
    _close(out2, stores.expected_decode(st2, q=q2.float().cpu().numpy()))


def test_a_mixed_batch_of_decodes_continuations_and_a_first_chunk_uses_every_path():
    w = _world(34, [70, 33, 50, 24], fresh=(3,))
    st = w["st"]
    md, raw_k, value, q = _step(w, [1, 1, 5, 24])
    key = torch.randn(sum([1, 1, 5, 24]), H, D, device="cuda").half()
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    out = _forward(impl, w, md, raw_k, value, q, key=key)
    sta = _after(w)
    qn = q.float().cpu().numpy()
    sub = dict(sta, block_table=sta["block_table"][:2], seq_lens=sta["seq_lens"][:2],
               decoders=sta["decoders"][:2])
    _close(out[:2], stores.expected_decode(sub, q=qn[:2]))
    _close(out[2:7], stores.expected_continuation(sta, 2, qn[2:7].transpose(1, 0, 2)).transpose(1, 0, 2))
    assert torch.isfinite(out[7:]).all()                      # the first chunk's SDPA rows
    assert rope_store.decoder_for_request(w["layer"].layer_name, int(st["block_table"][3][0])) is not None


def test_two_layers_of_one_step_each_write_and_read_their_own_store():
    w0 = _world(35, [60, 20], name="model.layers.0.self_attn.attn")
    w1 = _world(35, [60, 20], name="model.layers.1.self_attn.attn")
    md, raw_k, value, q = _step(w0, [1, 1])
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    o0 = _forward(impl, w0, md, raw_k, value, q)
    o1 = _forward(impl, w1, md, raw_k, value, q)              # same metadata object: plan reused
    for w, o in ((w0, o0), (w1, o1)):
        _close(o, stores.expected_decode(_after(w), q=q.float().cpu().numpy()))


def test_decode_refuses_a_request_with_no_fitted_decoder():
    w = _world(36, [30, 12], fresh=(1,))
    md, raw_k, value, q = _step(w, [1, 1])
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    with pytest.raises(RuntimeError, match="no fitted decoder|first chunk"):
        _forward(impl, w, md, raw_k, value, q)


# ---------------------------------------------------------------- the device-planned decode step
def test_device_planned_decode_step_matches_the_host_planned_one(monkeypatch):
    from vllm_ttkv import impl as impl_mod
    w = _world(37, [70, 33, 129, 17])
    md, raw_k, value, q = _step(w, [1, 1, 1, 1])
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    before = w["page"].clone()
    out_host = _forward(impl, w, md, raw_k, value, q)
    page_host = w["page"].clone()
    w["page"].copy_(before)
    monkeypatch.setattr(impl_mod, "_DEVICE_PLAN", True)
    md2, _, _, _ = _step(w, [1, 1, 1, 1])
    out_dev = _forward(impl, w, md2, raw_k, value, q)
    assert isinstance(getattr(md2, impl_mod._PLAN_ATTR), impl_mod.DevicePlan)
    assert torch.equal(w["page"], page_host)                   # the same bytes written
    # the read's bound differs (the table's rows), so the shares may split differently
    assert (out_dev.float() - out_host.float()).abs().max().item() < 1e-3
    _close(out_dev, stores.expected_decode(_after(w), q=q.float().cpu().numpy()))


def test_a_captured_decode_step_replays_for_the_next_steps(monkeypatch):
    """The forward captured once in a CUDA graph (device plan, no readback) and replayed for two
    steps whose lengths, slots and tokens differ from the captured one's."""
    from vllm_ttkv import impl as impl_mod
    from vllm_ttkv import ops
    monkeypatch.setattr(impl_mod, "_DEVICE_PLAN", True)
    w = _world(38, [70, 33, 129, 17])
    st0, name = w["st"], w["layer"].layer_name
    steps = []
    for back, seed in ((2, 0), (1, 1), (0, 2)):                 # seq_lens - 2, - 1, seq_lens
        ws = dict(w, st=dict(st0, seq_lens=st0["seq_lens"] - back))
        steps.append((ws, _step(ws, [1, 1, 1, 1], seed=seed)))
    md0, k0, v0, q0 = steps[0][1]
    buf = dict(seq=md0.seq_lens.clone(), slots=md0.slot_mapping.clone(), k=k0.clone(),
               v=v0.clone(), q=q0.clone())
    md = metadata.TTKVAttentionMetadata(
        seq_lens=buf["seq"], slot_mapping=buf["slots"], block_table=md0.block_table.clone(),
        query_start_loc=md0.query_start_loc, query_start_loc_cpu=md0.query_start_loc_cpu,
        num_actual_tokens=4, ttkv_serial=metadata.next_serial())
    out = torch.zeros(4, HQ, D, dtype=torch.float16, device="cuda")
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)

    def fwd():
        patch.stash_raw_k(name, buf["k"], None, w["table"])
        impl.forward(w["layer"], buf["q"], None, buf["v"], w["page"], md, out)

    ops.reset_status()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):                              # eager warm-up of the same path
        fwd()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fwd()
    for ws, (mds, ks, vs, qs) in steps[1:]:
        buf["seq"].copy_(mds.seq_lens)
        buf["slots"].copy_(mds.slot_mapping)
        buf["k"].copy_(ks)
        buf["v"].copy_(vs)
        buf["q"].copy_(qs)
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        _close(out, stores.expected_decode(_after(ws), q=qs.float().cpu().numpy()))
    ops.check_status()
    del graph


def test_device_plan_refuses_a_request_without_a_decoder_on_the_device(monkeypatch):
    from vllm_ttkv import impl as impl_mod
    from vllm_ttkv import ops
    monkeypatch.setattr(impl_mod, "_DEVICE_PLAN", True)
    w = _world(39, [30, 12], fresh=(1,))
    md, raw_k, value, q = _step(w, [1, 1])
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    ops.reset_status()
    out = _forward(impl, w, md, raw_k, value, q)
    with pytest.raises(RuntimeError, match="decoder"):
        ops.check_status()
    st = _after(w)
    sub = dict(st, block_table=st["block_table"][:1], seq_lens=st["seq_lens"][:1],
               decoders=st["decoders"][:1])
    _close(out[:1], stores.expected_decode(sub, q=q[:1].float().cpu().numpy()))


def test_a_device_planned_step_skips_the_padding_of_a_padded_batch(monkeypatch):
    """A decode batch padded to a captured size: the padding request has seq_len 0, slot
    PAD_SLOT_ID and no decoder. It writes and reads nothing and refuses nothing."""
    from vllm_ttkv import impl as impl_mod
    from vllm_ttkv import ops
    monkeypatch.setattr(impl_mod, "_DEVICE_PLAN", True)
    w = _world(41, [50, 23])
    md, raw_k, value, q = _step(w, [1, 1])
    pad = lambda t, v: torch.cat([t, torch.full_like(t[:1], v)])
    qsl = torch.arange(4, dtype=torch.int32)
    mdp = metadata.TTKVAttentionMetadata(
        seq_lens=pad(md.seq_lens, 0), slot_mapping=pad(md.slot_mapping, -1),
        block_table=pad(md.block_table, 0), query_start_loc=qsl.cuda(), query_start_loc_cpu=qsl,
        num_actual_tokens=3, ttkv_serial=metadata.next_serial())
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    rows = w["page"].view(-1, w["page"].shape[-1])             # [slots, blob]
    rows[md.slot_mapping] = 0xAB                               # the real tokens' slots, marked
    before = rows.clone()
    ops.reset_status()
    out = _forward(impl, w, mdp, pad(raw_k, 0), pad(value, 0), pad(q, 0))
    ops.check_status()
    assert torch.all(out[2] == 0)
    changed = (rows != before).any(1).nonzero().flatten().tolist()
    assert sorted(changed) == sorted(md.slot_mapping.tolist())  # the two real tokens' slots only
    _close(out[:2], stores.expected_decode(_after(w), q=q.float().cpu().numpy()))


def test_a_pinned_pool_refuses_to_grow():
    from vllm_ttkv import ops
    w = _world(40, [20])
    pool = rope_store.pool_for_layer(w["layer"].layer_name, w["lay"], "cuda")
    pool.pin()
    with pytest.raises(RuntimeError, match="reserve_rows"):
        pool._grow(pool.capacity + 1)
    ops._PINNED.pop(pool.decoders.data_ptr())


# ---------------------------------------------------------------- decoder lifetime and memory
def _rows(w, rows, seq_lens=None):
    """A view of world `w` holding only requests `rows` (in that order)."""
    st = dict(w["st"])
    st["block_table"] = st["block_table"][rows]
    st["seq_lens"] = st["seq_lens"][rows] if seq_lens is None else np.array(seq_lens, np.int32)
    st["decoders"] = st["decoders"][rows]
    st["pinvT"] = st["pinvT"][rows]
    st["kv"] = [st["kv"][r] for r in rows]
    return dict(w, st=st)


def test_a_finished_requests_pool_row_goes_to_the_next_request_which_reads_correctly():
    """Request 1 finishes and is released (the engine's completion hook); request 2's first chunk
    then gets request 1's pool row, and a decode step over requests 0 and 2 reads each request's
    own decoder from the pool."""
    from vllm_ttkv import metadata as md_mod
    w = _world(42, [70, 33, 41], fresh=(2,))
    st = w["st"]
    keys = [int(st["block_table"][r][0]) for r in range(3)]
    s1 = rope_store.request_slot(keys[1])
    assert s1 is not None and rope_store.request_slot(keys[2]) is None
    md_mod.TTKVAttentionMetadataBuilder.release_finished([keys[1]])
    assert rope_store.request_slot(keys[1]) is None
    assert rope_store.decoder_for_request(w["layer"].layer_name, keys[1]) is None
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    # request 2's first chunk: positions 0..39 (its store holds room for one more token)
    w2 = _rows(w, [2], seq_lens=[40])
    md, raw_k, value, q = _step(w2, [40])
    _forward(impl, w2, md, raw_k, value, q, key=torch.randn(40, H, D, device="cuda").half())
    assert rope_store.request_slot(keys[2]) == s1                       # the freed row, reused
    kdec = rope_store.decoder_for_request(w["layer"].layer_name, keys[2])
    # a decode step of requests 0 and 2 (request 2 now at 41 tokens)
    w02 = _rows(w, [0, 2])
    md2, raw_k2, value2, q2 = _step(w02, [1, 1], seed=3)
    out = _forward(impl, w02, md2, raw_k2, value2, q2)
    sta = _after(w02)
    sta["decoders"] = np.stack([st["decoders"][0], kdec.decoder_f.cpu().numpy()])
    _close(out, stores.expected_decode(sta, q=q2.float().cpu().numpy()))


def test_a_decode_steps_peak_allocation_is_within_the_memory_accounting():
    """The scratch a real step allocates (torch's peak over the step, fresh library buffers) is
    covered by `memory.step_scratch_bytes`, and the accounting does not overstate it by more than
    the parts a decode step does not use (the fit's tail)."""
    from vllm_ttkv import memory, ops
    w = _world(44, [300, 170, 257, 90, 33, 401, 12, 128])
    md, raw_k, value, q = _step(w, [1] * 8)
    impl = TTKVAttentionImpl(HQ, D, SCALE, H)
    out = torch.empty(8, HQ, D, dtype=torch.float16, device="cuda")
    ops.status_word(torch.device("cuda", torch.cuda.current_device()))
    ops._WORKSPACE.clear()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    patch.stash_raw_k(w["layer"].layer_name, raw_k, None, w["table"])
    impl.forward(w["layer"], q, None, value, w["page"], md, out)
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    lay = w["lay"]
    predicted = memory.step_scratch_bytes([lay], 8, 1, int(w["st"]["seq_lens"].max()), HQ)
    fit = int(ops._lib.lib().ttkv_fit_tail_scratch_bytes(lay.r1, lay.H, lay.H, lay.d))
    print(f"decode step: peak {peak} B allocated, accounting {predicted} B (fit tail {fit} B)")
    slack = 3 * (1 << 16) + (1 << 20)          # the 64 KiB floor of each cached buffer, small tensors
    assert peak <= predicted + slack
    assert predicted - fit <= peak + slack
