"""Parity of the CUDA read path (decode + continuation) with the oracle, through the C ABI.

Stores are encoded on the CPU by the oracle (`oracle/stores.py`), so these tests check the read
kernels independently of the write kernels. Tolerance: 2e-3 max-abs on attention outputs (the
fp16-store bound of the reference's `north_star`), 1e-2 for the 4-bit ("campaign4x") store.
"""
import numpy as np
import pytest
import torch

from oracle import stores
from oracle import ttkv_oracle as O

pytestmark = pytest.mark.gpu

ATOL_FP16_STORE = 2e-3
ATOL_4BIT_STORE = 1e-2


def _dev(st, q=None):
    dev = "cuda"
    from vllm_ttkv import layout as L
    g = st["g"]
    lay = L.TTKLayout(H=g.H, d=g.d, r1=g.r1, qbits=g.qbits, res_k=g.res_k, res_bits=g.res_bits,
                      v_lanes=g.v_lanes, v_bits=g.v_bits)
    tdt = {"float16": torch.float16, "bfloat16": torch.bfloat16}[st["dtype"]]
    return dict(
        lay=lay,
        cache=torch.from_numpy(st["cache"]).to(dev),
        bt=torch.from_numpy(st["block_table"]).to(dev),
        seq=torch.from_numpy(st["seq_lens"]).to(dev),
        dec=torch.from_numpy(st["decoders"]).to(dev),
        idx=torch.arange(len(st["seq_lens"]), dtype=torch.int32, device=dev),
        table=torch.from_numpy(st["table"]).to(dev).to(tdt),
        q=torch.from_numpy(st["q"] if q is None else q).to(dev).to(tdt),
        tdt=tdt)


def _decode(st, out_dtype=torch.float32, head_lo=0, head_hi=None, q=None, scale=None, images=False):
    from vllm_ttkv import ops
    d = _dev(st, q)
    B, HQ, _ = d["q"].shape
    out = torch.zeros(B, HQ, 128, dtype=out_dtype, device="cuda")
    ops.reset_status()
    ops.decode_paged(d["lay"], d["cache"], st["block_size"], d["bt"], d["seq"], d["dec"], d["idx"],
                     d["table"], d["q"], 128 ** -0.5 if scale is None else scale, out,
                     int(st["seq_lens"].max()), head_lo, head_hi,
                     images=ops.decoder_image(d["lay"], d["dec"]) if images else None)
    ops.check_status()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("cfg,atol", [("safe", ATOL_FP16_STORE), ("tight", ATOL_FP16_STORE),
                                      ("campaign4x", ATOL_4BIT_STORE)])
def test_decode_matches_oracle_ragged_batch(cfg, atol):
    st = stores.make_store(1, [70, 33, 129, 1, 16], cfg=cfg, r1=32)
    got = _decode(st)
    want = stores.expected_decode(st)
    err = np.abs(got - want).max()
    assert err < atol, err
    assert err < 1e-4, f"fp32 reconstruction drifted: {err}"


@pytest.mark.parametrize("HQ", [8, 32, 56])
def test_decode_gqa_groups(HQ):
    st = stores.make_store(2, [45, 100], cfg="safe", r1=24, HQ=HQ)
    assert np.abs(_decode(st) - stores.expected_decode(st)).max() < 1e-4


def test_decode_fp16_and_bf16_outputs_and_tables():
    """A 16-bit output carries its own rounding (the reference rounds `row.to(output.dtype)`
    too, impl.py:493): compare against the oracle rounded to the same dtype, 2e-3 + 1 ulp."""
    st = stores.make_store(3, [80, 17], cfg="safe", r1=40, dtype="bfloat16")
    want = stores.expected_decode(st)
    for odt, name, ulp in ((torch.float16, "float16", 2.0 ** -10), (torch.bfloat16, "bfloat16", 2.0 ** -7)):
        got = _decode(st, out_dtype=odt)
        want_r = torch.from_numpy(want).to(odt).float().numpy()
        assert np.all(np.abs(got - want_r) <= ATOL_FP16_STORE + ulp * np.abs(want_r)), name


def test_decode_rank_sweep_including_multiples_of_16():
    """The reference's Triton kernel crashed on r1 multiples of 16 (krt_triton.py:35-43). Ranks up
    to 192 take the tensor-core kernel; 200 takes the fp32 kernel."""
    for r1 in (16, 33, 61, 64, 110, 143, 200):
        st = stores.make_store(4, [150, 31], cfg="safe", r1=r1)
        assert np.abs(_decode(st) - stores.expected_decode(st)).max() < 1e-4, r1


def test_decode_head_shard_writes_only_its_heads():
    st = stores.make_store(5, [64, 40], cfg="safe", r1=32)
    want = stores.expected_decode(st)
    got = _decode(st, head_lo=2, head_hi=5)
    G = 3
    np.testing.assert_allclose(got[:, 2 * G:5 * G], want[:, 2 * G:5 * G], atol=1e-4)
    assert np.all(got[:, :2 * G] == 0) and np.all(got[:, 5 * G:] == 0)


def test_decode_long_context_split_merge():
    st = stores.make_store(6, [2100], cfg="safe", r1=48)
    assert np.abs(_decode(st) - stores.expected_decode(st)).max() < 1e-4


def test_decoder_images_stage_the_same_operand_the_decode_builds():
    """ttkv_decoder_image converts each decoder once; a decode staging the image must give the
    same bits as one converting the fp32 decoder itself (one and three K atoms)."""
    for r1 in (32, 110, 143):
        st = stores.make_store(12, [300, 77, 129], cfg="safe", r1=r1)
        a = _decode(st)
        b = _decode(st, images=True)
        assert np.array_equal(a, b), r1
        assert np.abs(b - stores.expected_decode(st)).max() < 1e-4, r1


def test_decode_schedule_over_more_requests_than_one_scan_chunk():
    """520 short requests: the device-side schedule sums the batch's tiles 512 requests at a time,
    and most CTAs get runs that cross several (request, head) pairs."""
    lens = np.random.default_rng(8).integers(1, 300, 520)
    st = stores.make_store(8, lens, cfg="safe", r1=24)
    assert np.abs(_decode(st) - stores.expected_decode(st)).max() < 1e-4


def test_decode_block_size_one_cuts_shares_into_virtual_shares():
    """With one token per block a CTA's cached block-table slice covers only 3 tiles, so 4 x 2100
    tokens x 8 heads (544 tiles) cut each CTA's share in two."""
    st = stores.make_store(9, [2100, 2100, 1900, 2050], cfg="safe", r1=32, block_size=1)
    assert np.abs(_decode(st) - stores.expected_decode(st)).max() < 1e-4


def test_rotation_is_per_row_negative_control():
    """Reading with the angle table shifted by one position must change the scores a lot --
    the failure this path is shaped around is a silent mis-rotation (reference.py:1-30)."""
    st = stores.make_store(7, [90], cfg="safe", r1=32)
    good = _decode(st)
    shifted = dict(st)
    shifted["table"] = np.concatenate([st["table"][1:], st["table"][-1:]])
    bad = _decode(shifted)
    assert np.abs(good - bad).max() > 1e-2


def test_decode_over_reference_golden_store():
    """The reference's own encoded store and its own attend_raw_store output."""
    from conftest import GOLDEN
    s = dict(np.load(GOLDEN / "store_safe_recip.npz"))
    g = O.geometry_for_config("safe", int(s["fit_coeff_q"].shape[1]))
    blobs = np.concatenate([np.concatenate([s["k_slots"], s["v_slots"]], 1),
                            np.concatenate([s["fz_k_slots"], s["fz_v_slots"]], 1)])
    n = blobs.shape[0]
    bs = 16
    bt = np.arange((n + bs - 1) // bs, dtype=np.int32)[::-1].copy()[None]
    cache = np.zeros((bt.size * bs, g.blob_bytes), np.uint8)
    cache[O.block_slots(bt[0], n, bs)] = blobs
    dec = np.zeros((1, g.r1, 1024), np.float32)
    d0 = s["fit_dec_q"].astype(np.float32) * s["fit_dec_scale"].view(np.float16).astype(np.float32)[:, None]
    dec[0, :d0.shape[0]] = d0
    st = dict(g=g, cache=cache, block_table=bt, seq_lens=np.array([n], np.int32), decoders=dec,
              table=s["table"].astype(np.float32), q=s["q"].astype(np.float32)[None],
              block_size=bs, dtype="float16")
    got = _decode(st)[0]
    assert np.abs(got - s["attend"]).max() < 1e-4


def _queries(rng, shape, qdt):
    """Standard normal queries, exact in the query dtype (returned as float32)."""
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
    return x.to({"float16": torch.float16, "bfloat16": torch.bfloat16}[qdt]).float().numpy()


@pytest.mark.parametrize("images,qdt,seqs,q_lens", [
    (False, "float16", [70, 40, 129], [6, 1, 37]),
    (True, "float16", [70, 40, 129], [6, 1, 37]),
    (True, "bfloat16", [70, 40, 129], [6, 1, 37]),
    (True, "float16", [300, 130, 47], [100, 129, 47])])
def test_continuation_matches_oracle_causal(images, qdt, seqs, q_lens):
    """With the decoders' images the chunk runs on the tensor-core continuation (blocks of 128
    (query, head) rows: 100 queries x 3 heads span three blocks and queries 42 and 85 have heads in
    two blocks; 300 stored rows are three tiles; a chunk equal to its request is a prompt read);
    without them on the 8-row blocks of the decode."""
    from vllm_ttkv import ops
    st = stores.make_store(8, seqs, cfg="safe", r1=32)
    rng = np.random.default_rng(0)
    qs = [_queries(rng, (24, ql, 128), qdt) for ql in q_lens]
    d = _dev(st)
    flat = np.ascontiguousarray(np.concatenate([q.transpose(1, 0, 2) for q in qs]))   # [N, HQ, d]
    qt = torch.from_numpy(flat).cuda().to({"float16": torch.float16, "bfloat16": torch.bfloat16}[qdt])
    start = np.concatenate([[0], np.cumsum(q_lens)[:-1]]).astype(np.int32)
    out = torch.zeros(qt.shape, dtype=torch.float32, device="cuda")
    ops.reset_status()
    ops.prefill_cont_paged(d["lay"], d["cache"], st["block_size"], d["bt"], d["seq"], d["dec"],
                           d["idx"], d["table"], torch.from_numpy(start).cuda(),
                           torch.tensor(q_lens, dtype=torch.int32, device="cuda"), qt,
                           128 ** -0.5, out, max(q_lens), int(st["seq_lens"].max()),
                           images=ops.decoder_image(d["lay"], d["dec"]) if images else None)
    ops.check_status()
    got = out.cpu().numpy()
    for r, ql in enumerate(q_lens):
        want = stores.expected_continuation(st, r, qs[r])                # [HQ, Q, d]
        err = np.abs(got[start[r]:start[r] + ql].transpose(1, 0, 2) - want).max()
        assert err < 1e-4, (r, err)


@pytest.mark.parametrize("images", [False, True])
@pytest.mark.parametrize("HQ,block_size,r1,cfg,q_lens", [
    (56, 16, 32, "safe", [20, 3]), (24, 1, 32, "safe", [20, 3]), (8, 16, 32, "safe", [20, 3]),
    (24, 16, 200, "safe", [20, 3]), (24, 16, 48, "campaign4x", [20, 3]), (24, 16, 32, "safe", [0, 11]),
    (24, 16, 126, "safe", [20, 3]), (24, 16, 14, "safe", [20, 3])])
def test_continuation_other_groups_block_sizes_and_ranks(HQ, block_size, r1, cfg, q_lens, images):
    """Without images: blocks of 8 (query, head) rows on the tensor-core decode for G = 7 (a block
    ends inside a query) and G = 1 (8 queries per block); one token per block sizes the plan
    beyond the default workspace, so the fp32 kernel serves unless the workspace holds it. With
    images: the tensor-core continuation (128 (query, head) rows per block: 20 queries x 7 heads
    are two blocks, the first ending inside query 18; 128 queries x 1 head).
    r1 = 200 is beyond both and takes the fp32 kernel; r1 = 126 is the continuation's largest
    rank, r1 = 14 a one-chunk coefficient block; the 4-bit store; a request with no queries."""
    from vllm_ttkv import ops
    st = stores.make_store(17, [90, 50], cfg=cfg, r1=r1, HQ=HQ, block_size=block_size)
    rng = np.random.default_rng(3)
    qs = [rng.standard_normal((HQ, ql, 128)).astype(np.float16).astype(np.float32) for ql in q_lens]
    d = _dev(st)
    flat = np.ascontiguousarray(np.concatenate([q.transpose(1, 0, 2) for q in qs]))
    qt = torch.from_numpy(flat).cuda().to(torch.float16)
    start = np.concatenate([[0], np.cumsum(q_lens)[:-1]]).astype(np.int32)
    out = torch.zeros(qt.shape, dtype=torch.float32, device="cuda")
    ops.reset_status()
    ops.prefill_cont_paged(d["lay"], d["cache"], block_size, d["bt"], d["seq"], d["dec"], d["idx"],
                           d["table"], torch.from_numpy(start).cuda(),
                           torch.tensor(q_lens, dtype=torch.int32, device="cuda"), qt, 128 ** -0.5,
                           out, max(q_lens), int(st["seq_lens"].max()),
                           images=ops.decoder_image(d["lay"], d["dec"]) if images else None)
    ops.check_status()
    got = out.cpu().numpy()
    for r, ql in enumerate(q_lens):
        if ql == 0:
            continue
        want = stores.expected_continuation(st, r, qs[r])
        assert np.abs(got[start[r]:start[r] + ql].transpose(1, 0, 2) - want).max() < 1e-4, (HQ, r)


def test_continuation_with_one_query_equals_decode():
    from vllm_ttkv import ops
    st = stores.make_store(9, [77, 12], cfg="safe", r1=32)
    d = _dev(st)
    dec = _decode(st)
    out = torch.zeros(2, 24, 128, device="cuda")
    ops.prefill_cont_paged(d["lay"], d["cache"], st["block_size"], d["bt"], d["seq"], d["dec"],
                           d["idx"], d["table"], torch.tensor([0, 1], dtype=torch.int32, device="cuda"),
                           torch.ones(2, dtype=torch.int32, device="cuda"), d["q"], 128 ** -0.5, out,
                           1, 77)
    np.testing.assert_allclose(out.cpu().numpy(), dec, atol=1e-5)   # two different kernels


def test_block_outside_the_cache_is_refused_on_device():
    from vllm_ttkv import ops
    st = stores.make_store(10, [40], cfg="safe", r1=32)
    bad = dict(st)
    bad["block_table"] = st["block_table"].copy()
    bad["block_table"][0, 1] = 10_000                                     # past the cache
    with pytest.raises(IndexError):
        _decode(bad)
    ops.reset_status()
    assert np.abs(_decode(st) - stores.expected_decode(st)).max() < 1e-4   # context still usable


def test_decoder_index_outside_pool_is_refused_on_device():
    from vllm_ttkv import ops
    st = stores.make_store(11, [20], cfg="safe", r1=32)
    d = _dev(st)
    out = torch.zeros(1, 24, 128, device="cuda")
    ops.reset_status()
    ops.decode_paged(d["lay"], d["cache"], 16, d["bt"], d["seq"], d["dec"],
                     torch.tensor([5], dtype=torch.int32, device="cuda"), d["table"], d["q"],
                     0.1, out, 20)
    with pytest.raises(RuntimeError, match="decoder"):
        ops.check_status()


def test_decode_refuses_a_request_longer_than_the_bound_on_device():
    from vllm_ttkv import ops
    st = stores.make_store(13, [300, 40], cfg="safe", r1=32)
    d = _dev(st)
    out = torch.zeros(2, 24, 128, device="cuda")
    ops.reset_status()
    ops.decode_paged(d["lay"], d["cache"], st["block_size"], d["bt"], d["seq"], d["dec"], d["idx"],
                     d["table"], d["q"], 128 ** -0.5, out, 100)
    with pytest.raises(RuntimeError, match="bound"):
        ops.check_status()
    want = stores.expected_decode(st)
    assert np.abs(out[1].cpu().numpy() - want[1]).max() < 1e-4            # within the bound: read


def test_decode_bound_far_above_the_batch_gives_the_same_result():
    """A graph captured with a large bound (the RoPE table's rows) replays shorter batches: the
    grid is one CTA per SM either way and only the workspace grows."""
    st = stores.make_store(14, [300, 77, 129], cfg="safe", r1=32)
    from vllm_ttkv import ops
    d = _dev(st)
    outs = []
    for bound in (300, int(st["table"].shape[0])):
        out = torch.zeros(3, 24, 128, device="cuda")
        ops.reset_status()
        ops.decode_paged(d["lay"], d["cache"], st["block_size"], d["bt"], d["seq"], d["dec"],
                         d["idx"], d["table"], d["q"], 128 ** -0.5, out, bound)
        ops.check_status()
        outs.append(out.cpu().numpy())
    assert np.abs(outs[0] - outs[1]).max() < 1e-5
    assert np.abs(outs[1] - stores.expected_decode(st)).max() < 1e-4


def test_decode_three_virtual_shares_per_cta():
    """One token per block: a segment may span 3 tiles, so 7 x 2100 tokens x 8 heads (952 tiles)
    cut each CTA's share into 3 virtual shares."""
    st = stores.make_store(15, [2100] * 7, cfg="safe", r1=24, block_size=1)
    assert np.abs(_decode(st) - stores.expected_decode(st)).max() < 1e-4


def test_decode_of_a_storage_shard_matches_the_full_decode_on_its_heads():
    """A shard's cache (its heads' rows), its decoders' columns and its heads' queries: the same
    outputs as the full store's decode on those heads (the schedules split differently, so to
    float rounding of the merge)."""
    from vllm_ttkv import ops
    from vllm_ttkv.layout import shard_slots
    st = stores.make_store(16, [300, 77, 129], cfg="safe", r1=110)
    d = _dev(st)
    full = _decode(st)
    G = 3
    for lo, hi in ((0, 4), (4, 8), (6, 8)):
        lay = d["lay"].shard(lo, hi)
        cache = shard_slots(d["cache"], d["lay"], lo, hi)
        dec = d["dec"][:, :, lo * 128:hi * 128].contiguous()
        q = d["q"][:, lo * G:hi * G]
        out = torch.zeros(3, (hi - lo) * G, 128, device="cuda")
        ops.reset_status()
        ops.decode_paged(lay, cache, st["block_size"], d["bt"], d["seq"], dec, d["idx"], d["table"],
                         q, 128 ** -0.5, out, int(st["seq_lens"].max()),
                         images=ops.decoder_image(lay, dec))
        ops.check_status()
        assert np.abs(out.cpu().numpy() - full[:, lo * G:hi * G]).max() < 1e-5, (lo, hi)


def test_continuation_paths_agree():
    """The 8-row blocks of the decode (no images) and the tensor-core continuation (images) on the
    same chunk: both within the kernel bound of the oracle, and within it of each other."""
    from vllm_ttkv import ops
    st = stores.make_store(18, [140, 60], cfg="safe", r1=110)
    q_lens = [33, 4]
    rng = np.random.default_rng(4)
    qs = [rng.standard_normal((24, ql, 128)).astype(np.float16).astype(np.float32) for ql in q_lens]
    d = _dev(st)
    qt = torch.from_numpy(np.ascontiguousarray(np.concatenate([q.transpose(1, 0, 2) for q in qs]))).cuda().half()
    start = torch.tensor([0, q_lens[0]], dtype=torch.int32, device="cuda")
    ql = torch.tensor(q_lens, dtype=torch.int32, device="cuda")
    outs = []
    for images in (None, ops.decoder_image(d["lay"], d["dec"])):
        out = torch.zeros(qt.shape, dtype=torch.float32, device="cuda")
        ops.reset_status()
        ops.prefill_cont_paged(d["lay"], d["cache"], 16, d["bt"], d["seq"], d["dec"], d["idx"], d["table"],
                               start, ql, qt, 128 ** -0.5, out, max(q_lens), int(st["seq_lens"].max()),
                               images=images)
        ops.check_status()
        outs.append(out.cpu().numpy())
    assert np.abs(outs[0] - outs[1]).max() < 1e-4
    for r, n in enumerate(q_lens):
        want = stores.expected_continuation(st, r, qs[r])
        s0 = int(start[r])
        for o in outs:
            assert np.abs(o[s0:s0 + n].transpose(1, 0, 2) - want).max() < 1e-4
