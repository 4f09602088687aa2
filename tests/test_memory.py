"""Memory accounting for an engine's profiling pass (`vllm_ttkv.memory`), on the CPU: the library's
sizing functions are host code."""
from vllm_ttkv import memory
from vllm_ttkv import synthetic as S
from vllm_ttkv.layout import layout_for_config


def _layers(cfg="safe"):
    return [layout_for_config(cfg, r1) for r1 in S.LLAMA32_3B_R1]


def test_cache_bytes_per_token_is_the_formats():
    assert memory.cache_bytes_per_token(_layers("safe")) == 25328       # the reference's README
    assert memory.cache_bytes_per_token(_layers("campaign4x")) == 25520


def test_scratch_and_pools_grow_with_the_step_and_the_requests():
    lays = _layers()
    small = memory.step_scratch_bytes(lays, 8, 1, 4323, 24)
    long_ = memory.step_scratch_bytes(lays, 8, 1, 16384, 24)
    chunked = memory.step_scratch_bytes(lays, 8, 256, 16384, 24)
    assert 0 < small <= long_ <= chunked
    one = memory.decoder_pool_bytes(lays, 1)
    assert memory.decoder_pool_bytes(lays, 64) == 64 * one
    # per request and layer: decoder + pinv (2 x r1 x 1024 x 4 B) and the operand image
    assert one > 2 * sum(S.LLAMA32_3B_R1) * 1024 * 4


def test_tokens_that_fit_sets_the_rest_aside():
    lays = _layers()
    free = 100 * 2 ** 30
    n = memory.tokens_that_fit(lays, free, 64, 256, 16384, 24)
    taken = memory.step_scratch_bytes(lays, 64, 256, 16384, 24) + memory.decoder_pool_bytes(lays, 64)
    per = memory.cache_bytes_per_token(lays)
    assert n == (free - taken) // per and n > 3_000_000
    assert memory.tokens_that_fit(lays, 1000, 64, 256, 16384, 24) == 0


def test_the_tensor_core_continuation_takes_no_scratch():
    lays = _layers()
    bound = memory.step_scratch_bytes(lays, 8, 256, 16384, 24)
    tc = memory.step_scratch_bytes(lays, 8, 256, 16384, 24, tc_continuation=True)
    decode_only = memory.step_scratch_bytes(lays, 8, 1, 16384, 24, max_tokens=8 * 256)
    # the calibrated layers above the continuation kernel's largest rank (130..143) still count
    # the 8-row plan's workspace, and they set the maximum
    assert any(l.r1 > memory.TC_CONTINUATION_MAX_R1 for l in lays)
    assert decode_only < tc <= bound
    small = [layout_for_config("safe", r) for r in (14, 67, 110, 126)]
    small_tc = memory.step_scratch_bytes(small, 8, 256, 16384, 24, tc_continuation=True)
    assert small_tc == memory.step_scratch_bytes(small, 8, 1, 16384, 24, max_tokens=8 * 256)
    assert small_tc < memory.step_scratch_bytes(small, 8, 256, 16384, 24)
    assert all(memory.tc_continuation_serves(l, 24) for l in small)
    assert not memory.tc_continuation_serves(layout_for_config("safe", 130), 24)
    assert not memory.tc_continuation_serves(layout_for_config("safe", 110), 80)     # G = 10
    assert not memory.tc_continuation_serves(layout_for_config("safe", 110), 20)     # HQ % H != 0
