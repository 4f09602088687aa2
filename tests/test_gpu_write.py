"""Parity of the CUDA write path (select/pack, frozen encode, fit tail) through the C ABI.

The bar is the reference's: slot bytes, bitmaps and codes are compared for EQUALITY. Where the
coefficients pass through an fp32 dot product whose summation order differs from the
reference's BLAS (the frozen projection and the residual reconstruction), the exact check is made
by feeding both sides the same fp32 coefficients; the end-to-end check reports the byte mismatch
rate and requires decoded values to agree.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import stores
from oracle import ttkv_oracle as O
from vllm_ttkv import synthetic as S

pytestmark = pytest.mark.gpu


def _lay(g):
    from vllm_ttkv.layout import TTKLayout
    return TTKLayout(H=g.H, d=g.d, r1=g.r1, qbits=g.qbits, res_k=g.res_k, res_bits=g.res_bits,
                     v_lanes=g.v_lanes, v_bits=g.v_bits)


def _pack_rows_gpu(X, lanes, bits, dtype=torch.float32):
    """Pack rows X [rows, 128] as one head of `rows` tokens into a scratch cache; return the
    bitmap / packed / scale bytes."""
    from vllm_ttkv import ops
    rows = X.shape[0]
    pb = O.packed_row_bytes(lanes, bits)
    width = ((16 + pb + 2 + 15) // 16) * 16
    cache = torch.zeros(rows, width, dtype=torch.uint8, device="cuda")
    x = torch.from_numpy(X).cuda().to(dtype).contiguous()
    ops.reset_status()
    ops.select_pack_rows(cache, torch.arange(rows, device="cuda"), x, field_off=0, row_stride=0,
                         lanes=lanes, bits=bits, heads=1, d=128)
    ops.check_status()
    c = cache.cpu().numpy()
    return c[:, :16], c[:, 16:16 + pb], c[:, 16 + pb:18 + pb].copy().view(np.float16).reshape(rows)


def test_select_pack_matches_reference_golden_rows():
    r = dict(np.load(GOLDEN / "rows_recip.npz"))
    for key in r:
        if not key.startswith("X_"):
            continue
        tag = key[2:]
        k, bits = int(tag.split("_")[0]), int(tag.split("_")[1])
        bm, pk, sc = _pack_rows_gpu(r[key], k, bits)
        assert np.array_equal(bm, r[f"bitmap_{tag}"]), tag
        assert np.array_equal(pk, r[f"packed_{tag}"]), tag
        assert np.array_equal(sc.view(np.uint16), r[f"scale_{tag}"]), tag


@pytest.mark.parametrize("lanes,bits", [(81, 3), (32, 3), (45, 3), (64, 4), (1, 2), (128, 8), (7, 5)])
def test_select_pack_matches_oracle_including_ties(lanes, bits):
    rng = np.random.default_rng(lanes * 10 + bits)
    X = rng.standard_normal((64, 128)).astype(np.float32)
    X[5] = 0.0                                                       # all-zero row: ruler 1/(2^(b-1)-1)
    X[6] = np.round(X[6])                                            # heavy ties
    X[7] = S.round_to_dtype(X[7] * 3, "bfloat16")
    bm, pk, sc = _pack_rows_gpu(X, lanes, bits)
    obm, opk, osc = O.encode_rows(X, lanes, bits, "recip")            # lowest-index ties too
    assert np.array_equal(bm, obm) and np.array_equal(pk, opk) and np.array_equal(sc, osc)


def test_select_pack_reads_bf16_rows_exactly():
    rng = np.random.default_rng(3)
    X = S.round_to_dtype(rng.standard_normal((32, 128)).astype(np.float32) * 2, "bfloat16")
    bm, pk, sc = _pack_rows_gpu(X, 81, 3, torch.bfloat16)
    obm, opk, osc = O.encode_rows(X, 81, 3, "recip")
    assert np.array_equal(bm, obm) and np.array_equal(pk, opk) and np.array_equal(sc, osc)


@pytest.mark.parametrize("name", ["store_safe_recip", "store_campaign4x_recip", "store_tight_recip"])
def test_fit_tail_matches_reference_golden(name):
    from vllm_ttkv import ops
    s = dict(np.load(GOLDEN / f"{name}.npz"))
    budget = int(s["fit_coeff_q"].shape[1])
    G1 = torch.from_numpy(s["G1"][0]).cuda()
    G2 = torch.from_numpy(s["G2"]).cuda()
    G3 = torch.from_numpy(s["G3"][:, :, 0]).cuda()
    out = ops.fit_tail(G1, G2, G3, budget)
    assert np.array_equal(out["coeff_q"].cpu().numpy(), s["fit_coeff_q"])
    cs16 = out["coeff_scale"].half().cpu().numpy().view(np.uint16)
    assert np.array_equal(cs16, s["fit_coeff_scale"])
    dq = out["dec_q"].cpu().numpy()
    assert (dq == s["fit_dec_q"]).mean() > 0.9999, (dq != s["fit_dec_q"]).sum()
    assert np.array_equal(out["dec_scale"].cpu().numpy().view(np.uint16), s["fit_dec_scale"])


def _frozen_case(seed=0, n_tok=7, cfg="safe", r1=32, kv_dtype="float16"):
    st = stores.make_store(seed, [50, 30], cfg=cfg, r1=r1)
    g = st["g"]
    K, V = S.synth_kv(seed + 99, n_tok)
    K = S.round_to_dtype(K, kv_dtype)
    V = S.round_to_dtype(V, kv_dtype)
    tok_dec = np.arange(n_tok, dtype=np.int32) % 2
    return st, g, K, V, tok_dec


def _write_gpu(g, K, V, tok_dec, decoders, pinvT=None, cq=None, cs=None, kv_dtype=torch.float16,
               heads=None):
    from vllm_ttkv import ops
    n = K.shape[1]
    lay = _lay(g)
    blob = lay.shard(*heads).compressed_bytes_per_token() if heads else g.blob_bytes
    cache = torch.zeros(n + 3, blob + 16, dtype=torch.uint8, device="cuda")
    slots = torch.arange(n, dtype=torch.int64, device="cuda") + 2           # not starting at 0
    k = torch.from_numpy(K.transpose(1, 0, 2).copy()).cuda().to(kv_dtype)
    v = torch.from_numpy(V.transpose(1, 0, 2).copy()).cuda().to(kv_dtype)
    ops.reset_status()
    ops.write_paged(lay, cache, slots, k, v, torch.from_numpy(tok_dec).cuda(),
                    torch.from_numpy(decoders).cuda(),
                    pinvs=None if pinvT is None else torch.from_numpy(pinvT).cuda(),
                    coeff_q=None if cq is None else torch.from_numpy(cq).cuda(),
                    coeff_scale=None if cs is None else torch.from_numpy(cs).cuda(), heads=heads)
    ops.check_status()
    c = cache.cpu().numpy()
    assert not c[:2].any() and not c[n + 2:].any(), "wrote outside the named slots"
    assert not c[:, blob:].any(), "wrote past the blob"
    return c[2:n + 2, :blob]


def test_write_given_coefficients_is_bit_exact():
    """Fit path: the caller's codes and fp32 rulers; R and V are packed exactly as the oracle."""
    st, g, K, V, tok_dec = _frozen_case()
    # coefficients from the oracle's frozen projection (one decoder per token), rulers in fp32
    cqs, css = [], []
    for t in range(K.shape[1]):
        M = K[:, t].reshape(1, -1)                                   # [1, H*d], m = h*d + j
        cq_t, cs_t = O.quant_coeff(M @ st["pinvT"][tok_dec[t]].T, 8)
        cqs.append(cq_t[0])
        css.append(cs_t[0, 0])
    cq = np.stack(cqs).astype(np.int8)
    cs = np.array(css, np.float32)
    got = _write_gpu(g, K, V, tok_dec, st["decoders"], cq=cq, cs=cs)
    # oracle: R from the same codes / rulers with the same decoders
    want = []
    for t in range(K.shape[1]):
        d = st["decoders"][tok_dec[t]]
        kd = ((cq[t].astype(np.float32) * cs[t]) @ d).reshape(g.H, g.d)
        R = (K[:, t] - kd).astype(np.float32)
        want.append(O.build_slots(g, cq[t:t + 1], cs[t:t + 1].astype(np.float16), R, V[:, t:t + 1])[0])
    want = np.stack(want)
    # V rows and the coefficient block are exact; K residual rows depend on R, whose fp32 sum
    # order differs -> require near-total byte agreement and identical coefficient blocks
    assert np.array_equal(got[:, :g.coeff_bytes + 2], want[:, :g.coeff_bytes + 2])
    assert np.array_equal(got[:, g.v_offset:], want[:, g.v_offset:])
    assert (got == want).mean() > 0.995


@pytest.mark.parametrize("r1,n_tok", [(32, 9), (143, 9), (208, 9), (32, 200), (110, 200)])
def test_frozen_write_matches_oracle_end_to_end(r1, n_tok):
    """Up to 96 tokens with r1 <= 200: the fused cluster write; 208: its two slices exceed shared
    memory, and 200 tokens (a prefill chunk) are past its token limit, so the two-launch write
    (projection, then encode + pack) runs."""
    st, g, K, V, tok_dec = _frozen_case(seed=1, n_tok=n_tok, r1=r1)
    got = _write_gpu(g, K, V, tok_dec, st["decoders"], pinvT=st["pinvT"])
    want = []
    for t in range(K.shape[1]):
        d, pv = st["decoders"][tok_dec[t]], st["pinvT"][tok_dec[t]].T
        cq, cs, R = O.encode_frozen(K[:, t:t + 1], d, pv)
        want.append(O.build_slots(g, cq, cs, R, V[:, t:t + 1])[0])
    want = np.stack(want)
    assert np.array_equal(got[:, g.v_offset:], want[:, g.v_offset:])        # V: no matmul upstream
    mism = (got != want).mean()
    assert mism < 0.01, mism
    # decoded keys agree (the read of a slot written here)
    for t in range(K.shape[1]):
        d = st["decoders"][tok_dec[t]]
        kg = O.dense_k(g, got[t:t + 1, :g.k_slot_bytes], d)
        kw = O.dense_k(g, want[t:t + 1, :g.k_slot_bytes], d)
        assert np.abs(kg - kw).max() < 5e-2 * max(1.0, np.abs(kw).max())


def test_frozen_write_over_reference_golden():
    """The reference's encode_frozen + torch pack of 5 tokens against its fitted decoder."""
    for name in ("store_safe_recip", "store_campaign4x_recip", "store_tight_recip"):
        s = dict(np.load(GOLDEN / f"{name}.npz"))
        cfg = name.split("_")[1]
        g = O.geometry_for_config(cfg, int(s["fit_coeff_q"].shape[1]))
        n = s["k_slots"].shape[0]
        K = s["K"].astype(np.float32)[:, n:]
        V = s["V"].astype(np.float32)[:, n:]
        dec = np.zeros((1, g.r1, 1024), np.float32)
        d0 = s["fit_dec_q"].astype(np.float32) * s["fit_dec_scale"].view(np.float16).astype(np.float32)[:, None]
        dec[0, :d0.shape[0]] = d0
        pinvT = s["pinv"].T[None].copy()
        got = _write_gpu(g, K, V, np.zeros(K.shape[1], np.int32), dec, pinvT=pinvT)
        want = np.concatenate([s["fz_k_slots"], s["fz_v_slots"]], 1)
        assert np.array_equal(got[:, g.v_offset:], want[:, g.v_offset:]), name
        assert np.array_equal(got[:, :g.coeff_bytes], want[:, :g.coeff_bytes]), name
        assert (got == want).mean() > 0.99, name


def test_write_refuses_pad_slot_on_device():
    from vllm_ttkv import ops
    st, g, K, V, tok_dec = _frozen_case(seed=2, n_tok=3)
    cache = torch.zeros(8, g.blob_bytes, dtype=torch.uint8, device="cuda")
    slots = torch.tensor([0, -1, 2], dtype=torch.int64, device="cuda")
    k = torch.from_numpy(K.transpose(1, 0, 2).copy()).cuda().half()
    v = torch.from_numpy(V.transpose(1, 0, 2).copy()).cuda().half()
    ops.reset_status()
    ops.write_paged(_lay(g), cache, slots, k, v, torch.from_numpy(tok_dec).cuda(),
                    torch.from_numpy(st["decoders"]).cuda(), pinvs=torch.from_numpy(st["pinvT"]).cuda())
    with pytest.raises(IndexError):
        ops.check_status()


@pytest.mark.parametrize("r1", [32, 208])
def test_write_skips_pad_slots_when_asked(r1):
    """TTKV_CACHE_SKIP_PAD (the padding of a batch padded to a captured graph): the padding tokens
    write nothing, even with a decoder row of -1, and the others write what they write alone
    (r1 32: the fused cluster write; 208: the two-launch write)."""
    from vllm_ttkv import ops
    st, g, K, V, tok_dec = _frozen_case(seed=3, n_tok=4, r1=r1)
    k = torch.from_numpy(K.transpose(1, 0, 2).copy()).cuda().half()
    v = torch.from_numpy(V.transpose(1, 0, 2).copy()).cuda().half()
    dec, pinv = torch.from_numpy(st["decoders"]).cuda(), torch.from_numpy(st["pinvT"]).cuda()
    rows = torch.from_numpy(tok_dec).cuda()
    rows_pad = rows.clone()
    rows_pad[1] = -1
    outs = []
    for slots, tdec, skip in (([0, 1, 2, 3], rows, False), ([0, -1, 2, -1], rows_pad, True)):
        cache = torch.full((8, g.blob_bytes), 7, dtype=torch.uint8, device="cuda")
        ops.reset_status()
        ops.write_paged(_lay(g), cache, torch.tensor(slots, dtype=torch.int64, device="cuda"), k, v,
                        tdec, dec, pinvs=pinv, skip_pad=skip)
        ops.check_status()
        outs.append(cache.cpu().numpy())
    full, padded = outs
    assert np.array_equal(padded[[0, 2]], full[[0, 2]])
    assert np.all(padded[[1, 3]] == 7) and np.all(padded[4:] == 7)


@pytest.mark.parametrize("r1", [32, 110, 208])
def test_storage_sharded_writes_reassemble_to_the_full_write(r1):
    """Each of 2, 4 and 8 shards written on its own (only its heads' rows, every head projected)
    reassembles to the bytes of the full write, bit for bit: the fused cluster write (r1 32, 110)
    and the two-launch write (208), frozen path; and the fit path with given coefficients."""
    import torch as _t
    from vllm_ttkv.layout import unshard_slots
    from vllm_ttkv.shard import head_range
    st, g, K, V, tok_dec = _frozen_case(seed=5, n_tok=6, r1=r1)
    lay = _lay(g)
    cases = {"frozen": dict(pinvT=st["pinvT"])}
    if r1 == 32:
        cq = np.random.default_rng(1).integers(-128, 128, (K.shape[1], r1)).astype(np.int8)
        cases["fit"] = dict(cq=cq, cs=np.full(K.shape[1], 0.013, np.float32))
    for name, kw in cases.items():
        full = _write_gpu(g, K, V, tok_dec, st["decoders"], **kw)
        for world in (2, 4, 8):
            ranges = [head_range(r, world, g.H) for r in range(world)]
            shards = [_t.from_numpy(_write_gpu(g, K, V, tok_dec, st["decoders"], heads=hr, **kw))
                      for hr in ranges]
            got = unshard_slots(shards, lay, ranges).numpy()
            assert np.array_equal(got, full), (name, world)


def test_write_then_read_round_trip():
    """A store written by the CUDA writer reads back (CUDA reader) like the oracle reads it."""
    from vllm_ttkv import ops
    st = stores.make_store(12, [65], cfg="safe", r1=32)
    g = st["g"]
    K, V = S.synth_kv(77, 5)
    cache = torch.from_numpy(st["cache"]).cuda()
    slots = O.block_slots(st["block_table"][0], 65, 16)[60:]             # overwrite the last 5
    k = torch.from_numpy(K.transpose(1, 0, 2).copy()).cuda().half()
    v = torch.from_numpy(V.transpose(1, 0, 2).copy()).cuda().half()
    ops.reset_status()
    ops.write_paged(_lay(g), cache, torch.from_numpy(slots).cuda(), k, v,
                    torch.zeros(5, dtype=torch.int32, device="cuda"),
                    torch.from_numpy(st["decoders"]).cuda(), pinvs=torch.from_numpy(st["pinvT"]).cuda())
    ops.check_status()
    st2 = dict(st)
    st2["cache"] = cache.cpu().numpy()
    assert not np.array_equal(st2["cache"], st["cache"])
    from test_gpu_read import _decode
    got = _decode(st2)
    want = stores.expected_decode(st2)
    assert np.abs(got - want).max() < 1e-4
