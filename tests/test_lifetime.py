"""Decoder lifetime on the CPU: a first chunk always refits (a finished request's decoder under the
same key is never reused), finished requests give their pool rows back, and the calibration table's
layer lookup. No GPU: the write's encoder calls are recorded, not run."""
import json
from types import SimpleNamespace

import pytest
import torch

from vllm_ttkv import impl as impl_mod
from vllm_ttkv import metadata, patch, rope_store
from vllm_ttkv.impl import StepPlan, TTKVAttentionImpl
from vllm_ttkv.layout import TTKLayout, layout_for_config, config

LAY = TTKLayout(H=8, d=128, r1=32, qbits=8, res_k=81, res_bits=3, v_lanes=81, v_bits=3)


def _md(q_lens, seq_lens, bt):
    qsl = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0).tolist()), dtype=torch.int32)
    n = int(qsl[-1])
    return metadata.TTKVAttentionMetadata(
        seq_lens=torch.tensor(seq_lens, dtype=torch.int32), slot_mapping=torch.arange(n),
        block_table=bt, query_start_loc=qsl, query_start_loc_cpu=qsl, num_actual_tokens=n)


@pytest.fixture
def recorder(monkeypatch):
    calls = []
    fitted = SimpleNamespace(decoder="NEW")
    monkeypatch.setattr(impl_mod.encode, "fit_into_budget", lambda *a, **k: calls.append("fit") or fitted)
    monkeypatch.setattr(impl_mod.encode, "write_fitted", lambda *a, **k: calls.append("write_fitted"))
    monkeypatch.setattr(impl_mod.encode, "write_frozen", lambda *a, **k: calls.append("write_frozen"))
    monkeypatch.setattr(impl_mod, "register_decoder",
                        lambda name, key, dec, lay=None: calls.append(("register", key, dec)))
    monkeypatch.setattr(impl_mod, "pool_for_layer",
                        lambda *a, **k: SimpleNamespace(decoders=None, pinvT=None))
    yield calls
    rope_store.clear_stores()


def _write(md, n_tok, stale_keys):
    name = "model.layers.3.self_attn.attn"
    impl = TTKVAttentionImpl(24, 128, 128 ** -0.5, 8)
    layer = SimpleNamespace(layer_name=name, ttkv_layout=LAY,
                            rotary_emb=SimpleNamespace(cos_sin_cache=torch.zeros(64, 128)))
    patch.stash_raw_k(name, torch.zeros(n_tok, 8 * 128), None, torch.zeros(64, 128))
    plan = StepPlan(md, 16, 1024, 0)
    orig = impl_mod.decoder_for_request
    impl_mod.decoder_for_request = lambda nm, k: "STALE" if k in stale_keys else None
    try:
        impl._write(layer, name, LAY, torch.zeros(1024, LAY.compressed_bytes_per_token(), dtype=torch.uint8),
                    torch.zeros(n_tok, 8, 128), plan, md, torch.device("cpu"))
    finally:
        impl_mod.decoder_for_request = orig


def test_a_first_chunk_refits_even_when_its_key_holds_a_finished_requests_decoder(recorder):
    # request 0 decodes against its own decoder; request 1 is a NEW request whose first block (7)
    # used to be the first block of a finished request that still has a decoder registered
    bt = torch.tensor([[3, 4, 5], [7, 8, 9]], dtype=torch.int32)
    md = _md([1, 6], [40, 6], bt)
    with pytest.MonkeyPatch.context() as mp:
        mp.setattr(impl_mod, "request_slot", lambda k, create=False: 0)
        _write(md, 7, stale_keys={3, 7})
    assert "fit" in recorder and "write_fitted" in recorder
    assert ("register", 7, "NEW") in recorder            # the stale decoder is replaced
    assert "write_frozen" in recorder                     # request 0 still uses its own decoder


def test_a_continuation_without_a_decoder_is_still_refused(recorder):
    bt = torch.tensor([[7, 8, 9]], dtype=torch.int32)
    md = _md([4], [20], bt)
    with pytest.raises(RuntimeError, match="first chunk was never written"):
        _write(md, 4, stale_keys=set())


def test_release_returns_the_pool_row_for_the_next_request():
    rope_store.clear_decoders()
    try:
        s0 = rope_store.request_slot(11, create=True)
        s1 = rope_store.request_slot(12, create=True)
        rope_store._DECODERS[("a", 11)] = object()
        rope_store._DECODERS[("b", 11)] = object()
        rope_store._DECODERS[("a", 12)] = object()
        metadata.TTKVAttentionMetadataBuilder.release_finished([11])
        assert rope_store.live_keys() == {12}
        assert ("a", 11) not in rope_store._DECODERS and ("b", 11) not in rope_store._DECODERS
        assert rope_store.request_slot(13, create=True) == s0 != s1   # the freed row is reused
    finally:
        rope_store.clear_decoders()


def test_absence_reaper_releases_only_after_the_grace_period():
    rope_store.clear_decoders()
    try:
        for k in (1, 2):
            rope_store.request_slot(k, create=True)
            rope_store._DECODERS[("x", k)] = object()
        reaper = rope_store.AbsenceReaper(2)
        assert reaper.step([1, 2]) == []
        assert reaper.step([1]) == []            # 2 missed once
        assert reaper.step([1, 2]) == []         # back: the count restarts
        assert reaper.step([1]) == []
        assert reaper.step([1]) == [2]           # missed twice in a row
        assert rope_store.live_keys() == {1}
        assert rope_store.AbsenceReaper(0).step([]) == []     # off by default
    finally:
        rope_store.clear_decoders()


def test_calibration_table_lookup(tmp_path):
    art = {"r1": [14, 28, 143], "layers": 3, "heads": 8, "head_dim": 128, "corpus": "synthetic"}
    path = tmp_path / "cal.json"
    path.write_text(json.dumps(art))
    info = rope_store.load_calibration(path, "safe")
    assert info["corpus"] == "synthetic" and rope_store.calibration_info()["r1"] == [14, 28, 143]
    assert rope_store.layout_for_layer("model.layers.2.self_attn.attn") == layout_for_config(config("safe"), 143)
    assert rope_store.layout_for_layer("attn.1").r1 == 28           # last integer component
    assert rope_store.layout_for_layer("model.layers.9.self_attn.attn") is None
    assert rope_store.layout_for_layer("lm_head") is None and rope_store.layout_for_layer(None) is None
    assert rope_store.block_index("model.layers.12.mlp.layers_x") == 12
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps(dict(art, layers=4)))
    with pytest.raises(ValueError, match="3 ranks"):
        rope_store.load_calibration(bad, "safe")
