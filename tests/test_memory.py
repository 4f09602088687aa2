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
