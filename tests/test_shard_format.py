"""The storage-sharded slot format (KV-head tensor parallelism) on the CPU: its geometry against the
C library's, the shard / reassemble round trip, and the oracle's read of a shard against its read
of the full store. The reference has no multi-GPU path; parity for this format is "the shards
reassemble to the reference's slot bytes" and "a shard reads like its heads of the full store"."""
import numpy as np
import pytest
import torch

from oracle import stores
from oracle import ttkv_oracle as O
from vllm_ttkv.layout import layout_for_config, shard_slots, unshard_slots
from vllm_ttkv.shard import head_range


@pytest.mark.parametrize("cfg,r1", [("safe", 110), ("tight", 143), ("campaign4x", 14)])
def test_shard_geometry_matches_the_library(cfg, r1):
    lay = layout_for_config(cfg, r1)
    for world in (1, 2, 4, 8):
        for rank in range(world):
            lo, hi = head_range(rank, world, lay.H)
            sl = lay.shard(lo, hi)
            st = sl.abi()                                   # ttkv_layout_init with H' heads
            assert st.H == hi - lo and st.blob_bytes == sl.compressed_bytes_per_token()
            assert sl.coeff_bytes == lay.coeff_bytes and sl.k_row_bytes == lay.k_row_bytes
    # safe r1=110 on 2 GPUs: 110 + 2 + 4 x 49 -> 320 B of K, 4 x 49 -> 208 B of V
    assert layout_for_config("safe", 110).shard(0, 4).compressed_bytes_per_token() == 528
    with pytest.raises(ValueError):
        lay.shard(3, 3)


def test_shards_reassemble_to_the_full_blob():
    rng = np.random.default_rng(0)
    lay = layout_for_config("safe", 77)
    head = lay.coeff_bytes + 2
    full = torch.from_numpy(rng.integers(0, 256, (33, lay.compressed_bytes_per_token()), dtype=np.uint8))
    # the format's padding bytes are zero
    full[:, head + lay.H * lay.k_row_bytes:lay.k_slot_bytes] = 0
    full[:, lay.v_offset + lay.H * lay.v_row_bytes:] = 0
    for world in (1, 2, 4, 8):
        ranges = [head_range(g, world, lay.H) for g in range(world)]
        shards = [shard_slots(full, lay, lo, hi) for lo, hi in ranges]
        assert all(s.shape[1] == lay.shard(lo, hi).compressed_bytes_per_token()
                   for s, (lo, hi) in zip(shards, ranges))
        assert torch.equal(unshard_slots(shards, lay, ranges), full), world
    with pytest.raises(ValueError, match="exactly once"):
        unshard_slots([full], lay, [(0, 4)])


def test_a_shard_reads_like_its_heads_of_the_full_store():
    """The oracle's decode of a shard (H' heads, the decoders' columns of those heads, their query
    rows) equals its decode of the full store on those heads."""
    st = stores.make_store(21, [70, 19, 140], cfg="safe", r1=40)
    g = st["g"]
    lay = layout_for_config("safe", 40)
    full = O.decode_batch(g, st["cache"], st["block_table"], st["seq_lens"], st["block_size"],
                          st["q"], list(st["decoders"]), st["table"])
    G = st["q"].shape[1] // g.H
    for lo, hi in ((0, 4), (4, 8), (2, 3)):
        cache = shard_slots(torch.from_numpy(st["cache"]), lay, lo, hi).numpy()
        gs = O.geometry_for_config("safe", 40, H=hi - lo)
        dec = [d[:, lo * 128:hi * 128].copy() for d in st["decoders"]]
        got = O.decode_batch(gs, cache, st["block_table"], st["seq_lens"], st["block_size"],
                             st["q"][:, lo * G:hi * G].copy(), dec, st["table"])
        np.testing.assert_allclose(got, full[:, lo * G:hi * G], rtol=0, atol=1e-6)
