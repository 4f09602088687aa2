"""The vLLM-facing adapter on the CPU: refusals, the step plan, the raw-K hand-over and the metadata
(the reference's tests/test_impl_decode.py guards that need no GPU)."""
import pytest
import torch
from torch import nn

from vllm_ttkv import metadata, patch
from vllm_ttkv.impl import (DevicePlan, StepPlan, TTKVAttentionImpl, decode_only, plan_for,
                            validate_slot_ids)
from vllm_ttkv.layout import TTKLayout


def _md(q_lens, seq_lens, slots=None, bt=None, serial=0):
    qsl = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0).tolist()), dtype=torch.int32)
    n = int(qsl[-1])
    return metadata.TTKVAttentionMetadata(
        seq_lens=torch.tensor(seq_lens, dtype=torch.int32),
        slot_mapping=torch.arange(n, dtype=torch.int64) if slots is None else torch.tensor(slots),
        block_table=torch.arange(len(q_lens) * 4, dtype=torch.int32).reshape(len(q_lens), 4) if bt is None else bt,
        query_start_loc=qsl, query_start_loc_cpu=qsl, num_actual_tokens=n, ttkv_serial=serial)


def test_constructor_refuses_the_features_it_cannot_honour():
    for kw in ({"alibi_slopes": [1.0]}, {"logits_soft_cap": 30.0}, {"sliding_window": 128},
               {"kv_sharing_target_layer_name": "model.layers.0.self_attn.attn"}):
        with pytest.raises(NotImplementedError):
            TTKVAttentionImpl(24, 128, 128 ** -0.5, 8, **kw)
    with pytest.raises(ValueError):
        TTKVAttentionImpl(24, 128, 1.0, 7)


def test_refuses_fused_output_quantization_and_a_two_tensor_cache():
    impl = TTKVAttentionImpl(24, 128, 128 ** -0.5, 8)
    with pytest.raises(NotImplementedError):
        impl.forward(None, torch.zeros(1, 24, 128), None, None, None, None, torch.zeros(1, 24, 128),
                     output_scale=torch.ones(1))
    with pytest.raises(RuntimeError, match="ONE cache tensor"):
        impl._cache_tensor((torch.zeros(1), torch.zeros(1)))


def test_no_metadata_zeroes_the_output():
    impl = TTKVAttentionImpl(24, 128, 128 ** -0.5, 8)
    out = torch.ones(2, 24, 128)
    impl.forward(None, torch.zeros(2, 24, 128), None, None, None, None, out)
    assert not out.any()


def test_layout_head_dim_mismatch_refuses():
    impl = TTKVAttentionImpl(24, 64, 64 ** -0.5, 8)

    class L:
        layer_name = "model.layers.0.self_attn.attn"
        ttkv_layout = TTKLayout(H=8, d=128, r1=32, qbits=8, res_k=81, res_bits=3, v_lanes=81, v_bits=3)
    with pytest.raises(RuntimeError, match="head_dim"):
        impl._layout(L())


def test_plan_splits_decodes_from_prefills_and_reads_the_keys():
    md = _md([1, 1, 5, 3], [10, 20, 5, 30])
    p = StepPlan(md, 16, 1024, 0)
    assert p.n_dec == 2 and p.prefills == [2, 3] and p.qsl == [0, 1, 2, 7, 10]
    assert p.keys == [0, 4, 8, 12]
    assert p.seq_lens == [10, 20, 5, 30]


def test_refuses_a_batch_whose_decodes_are_not_at_the_front():
    with pytest.raises(RuntimeError, match="front of the batch"):
        StepPlan(_md([4, 1], [9, 7]), 16, 1024, 0)


def test_the_step_refuses_a_padded_or_out_of_range_slot_for_the_whole_step():
    with pytest.raises(RuntimeError, match="PAD_SLOT_ID"):
        StepPlan(_md([1, 1], [3, 3], slots=[5, -1]), 16, 1024, 0)
    with pytest.raises(IndexError):
        validate_slot_ids(torch.tensor([0, 2048]), 2, 1024)


def test_plan_is_reused_within_a_step_and_rebuilt_for_the_next():
    md = _md([1, 1], [3, 4], serial=metadata.next_serial())
    p1 = plan_for(md, 16, 1024)
    assert plan_for(md, 16, 1024) is p1
    md.ttkv_serial = metadata.next_serial()
    assert plan_for(md, 16, 1024) is not p1
    md.ttkv_serial = 0                                     # not built here: never cached
    assert plan_for(md, 16, 1024) is not plan_for(md, 16, 1024)


def test_decode_only_reads_the_host_copy_of_the_query_starts():
    assert decode_only(_md([1, 1, 1], [3, 4, 5])) == 3
    assert decode_only(_md([1, 2], [3, 4])) == 0
    assert decode_only(_md([0, 2], [3, 4])) == 0                  # the same total, not all ones
    md = _md([1, 1], [3, 4])
    md.query_start_loc_cpu = None
    assert decode_only(md) == 0


def test_a_device_plan_reads_nothing_back_and_defers_the_refusals():
    # a PAD_SLOT_ID slot is refused by the host plan before any launch ...
    md = _md([1, 1], [3, 3], slots=[5, -1], serial=metadata.next_serial())
    with pytest.raises(RuntimeError, match="PAD_SLOT_ID"):
        plan_for(md, 16, 1024)
    # ... and left to the kernels' status word by the device plan
    p = plan_for(md, 16, 1024, device_plan=True)
    assert isinstance(p, DevicePlan) and p.n == 2
    assert plan_for(md, 16, 1024, device_plan=True) is p
    assert plan_for(md, 16, 1024, device_plan=True, capturing=True) is not p   # captured anew
    # a step with a prefill keeps the host plan
    assert isinstance(plan_for(_md([1, 3], [3, 9]), 16, 1024, device_plan=True), StepPlan)


def test_the_device_key_map_follows_the_registry():
    from vllm_ttkv import ops, rope_store
    rope_store.clear_decoders()
    try:
        rope_store._REQ_SLOT.update({7: 0, 40: 3})
        lut = rope_store.key_rows("cpu", 64)
        assert lut.numel() >= 64 and int(lut[7]) == 0 and int(lut[40]) == 3 and int(lut[8]) == -1
        rope_store._set_key_row(1500, 5)                         # past the map: it grows
        rows = rope_store.rows_for_keys(torch.tensor([40, 7, 1500, 9, -1, 10 ** 7], dtype=torch.int32))
        assert rows.tolist() == [3, 0, 5, -1, -1, -1] and rows.dtype == torch.int32
        lut = rope_store.key_rows("cpu")
        ops.pin(lut)
        with pytest.raises(RuntimeError, match="reserve_keys"):
            rope_store.key_rows("cpu", lut.numel() + 1)
        rope_store.clear_decoders()                              # a pinned map is emptied, kept
        assert rope_store.key_rows("cpu") is lut and int(lut[40]) == -1
    finally:
        ops._PINNED.clear()
        rope_store.clear_decoders()


def test_metadata_build_copies_the_step_and_stamps_a_new_serial():
    class Common:
        seq_lens = torch.tensor([5], dtype=torch.int32)
        slot_mapping = torch.tensor([4])
        block_table_tensor = torch.zeros(1, 2, dtype=torch.int32)
        query_start_loc = torch.tensor([0, 1], dtype=torch.int32)
        query_start_loc_cpu = query_start_loc
        num_actual_tokens, max_query_len, max_seq_len = 1, 1, 5
    a, b = metadata.build(Common()), metadata.build(Common())
    assert a.block_table is Common.block_table_tensor and a.num_actual_tokens == 1
    assert 0 < a.ttkv_serial < b.ttkv_serial


def test_take_raw_k_pops_and_refuses_a_missing_or_doubled_capture():
    patch.clear_stash()
    with pytest.raises(RuntimeError, match="no raw K"):
        patch.take_raw_k("model.layers.0.self_attn.attn")
    patch.stash_raw_k("L0", torch.ones(1), None)
    with pytest.raises(RuntimeError, match="already waiting"):
        patch.stash_raw_k("L0", torch.ones(1), None)
    assert patch.take_raw_k("L0")["raw_k"].item() == 1.0
    with pytest.raises(RuntimeError):
        patch.take_raw_k("L0")


def test_install_wraps_each_rotary_call_and_stashes_the_raw_key():
    patch.clear_stash()

    class Rope(nn.Module):
        cos_sin_cache = torch.zeros(4, 128)

        def forward(self, positions, q, k):
            return q + 1, k + 1                              # "rotated"

    class Attn(nn.Module):
        layer_name = "model.layers.3.self_attn.attn"

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.rotary_emb, self.attn = Rope(), Attn()

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.block = Block()

    m = Model()
    assert patch.install(m) == 1
    q, k = m.block.rotary_emb(torch.arange(2), torch.zeros(2), torch.zeros(2))
    assert (k == 1).all()
    got = patch.take_raw_k("model.layers.3.self_attn.attn")
    assert (got["raw_k"] == 0).all() and got["cos_sin_cache"] is Rope.cos_sin_cache
    with pytest.raises(RuntimeError, match="no block"):
        patch.install(nn.Linear(2, 2))
