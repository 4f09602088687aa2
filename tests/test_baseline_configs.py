"""Parity at BASELINE's own configurations, at their full sizes.

  cfg 0  1 request x 1082 tokens, r1 = 110, `safe`, fp16 model: the store, the decoder and the
         attention output were produced by the REFERENCE itself (tests/golden/make_golden.py,
         `store_cfg0_recip.npz`); the oracle is pinned to it on the CPU, the CUDA read and write
         are compared with it on the GPU.
  cfg 1  one full layer of the decode step: 8 requests x 4322 tokens at the calibrated ranks 14,
         110 and 143, `safe`, bf16 model.
  cfg 2  a `campaign4x` ("4-bit") point at 14402 tokens (4 requests read, 2 checked).
  cfg 3  one 256-query continuation chunk over 7379 stored tokens (2 prompts).
  cfg 4  the encode of 16384 tokens at r1 = 110, `tight`: bit-exact slot bytes when the kernels
         get the oracle's fp32 inputs (cores, residual, V), and the per-field mismatch rates of
         the end-to-end encode from raw K.

Stores for cfg 1-3 are encoded on the GPU by this repository's encoder; the oracle reads the same
bytes with the same decoders, so these check the read at full size. Tolerances: attention outputs
2e-3 max-abs for an fp16 store and 1e-2 for the 4-bit one (the reference's bar); the read kernels
are also held to their own bound, 1e-4, where the output is fp32.
"""
import hashlib

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import ttkv_oracle as O
from vllm_ttkv import synthetic as S

ATOL_FP16_STORE = 2e-3
ATOL_4BIT_STORE = 1e-2
KERNEL_BOUND = 1e-4


def _sha(a):
    return np.frombuffer(hashlib.sha256(a.astype(np.float16).tobytes()).digest(), np.uint8)


def cfg0_case():
    """The golden store and its inputs: K, V regenerated from the seed (checked by SHA-256) with
    the reference's tie-breaking redraws of V applied."""
    s = dict(np.load(GOLDEN / "store_cfg0_recip.npz"))
    K, V = S.synth_kv(int(s["seed"]), int(s["n"]))
    K = S.round_to_dtype(K, "float16")
    V = S.round_to_dtype(V, "float16")
    assert np.array_equal(_sha(K), s["K_sha256"]) and np.array_equal(_sha(V), s["V_sha256"]), \
        "synth_kv no longer reproduces the inputs the golden store was made from"
    Vr = V.reshape(-1, 128)
    Vr[s["v_fix_rows"]] = s["v_fix"].astype(np.float32)
    g = O.geometry_for_config("safe", int(s["r1"]))
    dec = np.zeros((g.r1, g.H * g.d), np.float32)
    r = int(s["fit_rank"])
    dec[:r] = s["dec_q"].astype(np.float32) * s["dec_scale"].view(np.float16).astype(np.float32)[:, None]
    table = S.cos_sin_cache(int(s["n"]) + 6, dtype="float16")
    return s, g, K, V, dec, table


# ----------------------------------------------------------------------------- cfg 0, CPU pins
def test_cfg0_oracle_is_pinned_to_the_reference_at_full_size():
    s, g, K, V, dec, table = cfg0_case()
    n = K.shape[1]
    f = O.fit_into_budget(K, g, "safe", "recip", cores=(s["G1"], s["G2"], s["G3"]))
    assert f["fitted_rank"] == int(s["fit_rank"])
    assert np.array_equal(f["dec_q"], s["dec_q"])
    assert np.array_equal(f["dec_scale"].view(np.uint16), s["dec_scale"])
    blob = O.build_slots(g, f["coeff_q"], f["coeff_scale"], f["R"], V, "recip")
    ks, vs = blob[:, :g.k_slot_bytes], blob[:, g.k_slot_bytes:]
    cb = g.coeff_bytes + 2
    assert np.array_equal(ks[:, :cb], s["k_slots"][:, :cb]), "coefficient block"
    assert np.array_equal(vs, s["v_slots"]), "V slots"
    # the residual passes through an fp32 GEMM whose summation order is BLAS's
    assert (ks == s["k_slots"]).mean() > 0.999
    cos, sin = O.cos_sin_from_table(table, np.arange(n), 128)
    out = O.attend(g, s["k_slots"], s["v_slots"], dec, s["q"].astype(np.float32), cos, sin)
    np.testing.assert_allclose(out, s["attend"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(out, s["attend_oracle"], rtol=1e-5, atol=1e-5)


# ----------------------------------------------------------------------------- GPU helpers
def _lay(g):
    from vllm_ttkv.layout import TTKLayout
    return TTKLayout(H=g.H, d=g.d, r1=g.r1, qbits=g.qbits, res_k=g.res_k, res_bits=g.res_bits,
                     v_lanes=g.v_lanes, v_bits=g.v_bits)


def _paged(blobs_per_req, block_size=16, seed=0):
    """Scatter each request's blobs into a paged cache through a seeded random block table."""
    lens = [b.shape[0] for b in blobs_per_req]
    bt, nblk = S.block_table(seed, lens, block_size)
    cache = np.zeros((nblk * block_size, blobs_per_req[0].shape[1]), np.uint8)
    for r, b in enumerate(blobs_per_req):
        cache[O.block_slots(bt[r], lens[r], block_size)] = b
    return cache, bt


def _decode_gpu(lay, cache, bt, seq_lens, decoders, table, q, out_dtype, block_size=16):
    from vllm_ttkv import ops
    dev = "cuda"
    B, HQ, _ = q.shape
    out = torch.zeros(B, HQ, 128, dtype=out_dtype, device=dev)
    dec_t = torch.as_tensor(decoders).to(dev).contiguous()
    ops.reset_status()
    ops.decode_paged(lay, torch.as_tensor(cache).to(dev), block_size, torch.as_tensor(bt).to(dev),
                     torch.as_tensor(np.asarray(seq_lens, np.int32)).to(dev), dec_t,
                     torch.arange(B, dtype=torch.int32, device=dev), table, q, 128 ** -0.5, out,
                     int(max(seq_lens)), images=ops.decoder_image(lay, dec_t))
    ops.check_status()
    return out.float().cpu().numpy()


def _gpu_store(lens, r1, cfg, seed, dtype="bfloat16", block_size=16):
    """Requests of `lens` tokens encoded by this repository's GPU encoder (device fit + writer)
    into one paged cache; returns host copies of everything the oracle needs."""
    from vllm_ttkv import encode
    from vllm_ttkv.layout import config, layout_for_config
    lay = layout_for_config(config(cfg), r1)
    bt, nblk = S.block_table(seed, lens, block_size)
    cache = torch.zeros(nblk * block_size, lay.compressed_bytes_per_token(), dtype=torch.uint8, device="cuda")
    decs = np.zeros((len(lens), r1, 8 * 128), np.float32)
    for r, n in enumerate(lens):
        K, V = S.synth_kv(seed * 100 + r, n)
        K, V = S.round_to_dtype(K, dtype), S.round_to_dtype(V, dtype)
        Kt = torch.from_numpy(K).cuda()
        fk = encode.fit_into_budget(Kt, lay, cfg)
        slots = torch.from_numpy(O.block_slots(bt[r], n, block_size)).cuda()
        encode.write_fitted(cache, slots, fk, Kt.permute(1, 0, 2).contiguous(),
                            torch.from_numpy(V).cuda().permute(1, 0, 2).contiguous(), lay)
        decs[r] = fk.decoder.decoder_f.cpu().numpy()
    torch.cuda.synchronize()
    g = O.geometry_for_config(cfg, r1)
    return lay, g, cache, cache.cpu().numpy(), bt, decs


# ----------------------------------------------------------------------------- cfg 0, GPU
@pytest.mark.gpu
def test_cfg0_decode_matches_the_reference_output():
    s, g, K, V, dec, table_np = cfg0_case()
    lay = _lay(g)
    cache, bt = _paged([np.concatenate([s["k_slots"], s["v_slots"]], 1)], seed=3)
    table = torch.from_numpy(table_np).cuda().half()
    q = torch.from_numpy(s["q"]).cuda().view(1, 24, 128)
    want = s["attend"][None]
    got32 = _decode_gpu(lay, cache, bt, [K.shape[1]], dec[None], table, q, torch.float32)
    err = np.abs(got32 - want).max()
    assert err < KERNEL_BOUND, err
    got16 = _decode_gpu(lay, cache, bt, [K.shape[1]], dec[None], table, q, torch.float16)
    want16 = want.astype(np.float16).astype(np.float32)
    assert np.all(np.abs(got16 - want16) <= ATOL_FP16_STORE + 2.0 ** -10 * np.abs(want16))


@pytest.mark.gpu
def test_cfg0_write_reproduces_the_reference_slots():
    """The reference's SVD cores in, the whole 1082-token store out: the fit tail, the coefficient
    block and the V slots byte-exact; the K residual exact where its fp32 GEMM rounds alike."""
    from vllm_ttkv import encode, ops
    s, g, K, V, dec, _ = cfg0_case()
    lay = _lay(g)
    n = K.shape[1]
    G1 = torch.from_numpy(s["G1"][0]).cuda()
    G2 = torch.from_numpy(s["G2"]).cuda()
    G3 = torch.from_numpy(s["G3"][:, :, 0]).cuda()
    ft = ops.fit_tail(G1, G2, G3, g.r1)
    assert np.array_equal(ft["dec_q"].cpu().numpy(), s["dec_q"])
    assert np.array_equal(ft["dec_scale"].cpu().numpy().view(np.uint16), s["dec_scale"])
    fk = encode.FittedK(ft["coeff_q"], ft["coeff_scale"], encode.KDecoder(ft["decoder"]), ft["dec_q"],
                        ft["dec_scale"], int(s["fit_rank"]), g.r1)
    cache = torch.zeros(n, g.blob_bytes, dtype=torch.uint8, device="cuda")
    encode.write_fitted(cache, torch.arange(n, device="cuda"), fk,
                        torch.from_numpy(K).cuda().half().permute(1, 0, 2).contiguous(),
                        torch.from_numpy(V).cuda().half().permute(1, 0, 2).contiguous(), lay)
    c = cache.cpu().numpy()
    ks, vs = c[:, :g.k_slot_bytes], c[:, g.k_slot_bytes:]
    cb = g.coeff_bytes + 2
    assert np.array_equal(ks[:, :cb], s["k_slots"][:, :cb])
    assert np.array_equal(vs, s["v_slots"])
    rate = (ks != s["k_slots"]).mean()
    print(f"cfg0 K-slot byte mismatch rate vs the reference: {rate:.2e}")
    assert rate < 1e-3


# ----------------------------------------------------------------------------- cfg 1
@pytest.mark.gpu
@pytest.mark.parametrize("r1", [14, 110, 143])
def test_cfg1_full_layer_decode(r1):
    n = 4322
    lay, g, cache_t, cache, bt, decs = _gpu_store([n] * 8, r1, "safe", seed=r1)
    table_np = S.cos_sin_cache(n + 16, dtype="bfloat16")
    qn = S.synth_queries(r1, (8, 24, 128), "bfloat16")
    got = _decode_gpu(lay, cache, bt, [n] * 8, decs, torch.from_numpy(table_np).cuda().bfloat16(),
                      torch.from_numpy(qn).cuda().bfloat16(), torch.float32)
    want = O.decode_batch(g, cache, bt, [n] * 8, 16, qn, list(decs), table_np)
    err = np.abs(got - want).max()
    assert err < KERNEL_BOUND, err


# ----------------------------------------------------------------------------- cfg 2
@pytest.mark.gpu
def test_cfg2_campaign4x_at_14402_tokens():
    n, B = 14402, 4
    lay, g, cache_t, cache, bt, decs = _gpu_store([n] * B, 110, "campaign4x", seed=2)
    table_np = S.cos_sin_cache(n + 16, dtype="bfloat16")
    qn = S.synth_queries(2, (B, 24, 128), "bfloat16")
    got = _decode_gpu(lay, cache, bt, [n] * B, decs, torch.from_numpy(table_np).cuda().bfloat16(),
                      torch.from_numpy(qn).cuda().bfloat16(), torch.float32)
    want = O.decode_batch(g, cache, bt[:2], [n] * 2, 16, qn[:2], list(decs[:2]), table_np)
    err = np.abs(got[:2] - want).max()
    assert err < ATOL_4BIT_STORE and err < KERNEL_BOUND, err


# ----------------------------------------------------------------------------- cfg 3
@pytest.mark.gpu
def test_cfg3_continuation_chunk_of_256_queries_over_7379_tokens():
    from vllm_ttkv import ops
    n, Q, B = 7379, 256, 2
    lay, g, cache_t, cache, bt, decs = _gpu_store([n] * B, 110, "safe", seed=3, dtype="float16")
    table_np = S.cos_sin_cache(n + 16, dtype="float16")
    qm = S.synth_queries(3, (B, Q, 24, 128), "float16")
    dev = "cuda"
    out = torch.zeros(B * Q, 24, 128, dtype=torch.float32, device=dev)
    dec_t = torch.from_numpy(decs).cuda()
    ops.reset_status()
    ops.prefill_cont_paged(lay, cache_t, 16, torch.from_numpy(bt).cuda(),
                           torch.full((B,), n, dtype=torch.int32, device=dev), dec_t,
                           torch.arange(B, dtype=torch.int32, device=dev),
                           torch.from_numpy(table_np).cuda().half(),
                           torch.tensor([0, Q], dtype=torch.int32, device=dev),
                           torch.full((B,), Q, dtype=torch.int32, device=dev),
                           torch.from_numpy(qm.reshape(B * Q, 24, 128)).cuda().half(), 128 ** -0.5,
                           out, Q, n, images=ops.decoder_image(lay, dec_t))
    ops.check_status()
    got = out.cpu().numpy().reshape(B, Q, 24, 128)
    cos, sin = O.cos_sin_from_table(table_np, np.arange(n), 128)
    for r in range(B):
        slots = O.block_slots(bt[r], n, 16)
        ks, vs = O.read_blob(cache, slots, g)
        want = O.attend_multi(g, ks, vs, decs[r], qm[r].transpose(1, 0, 2), cos, sin, p0=n - Q)
        err = np.abs(got[r] - want.transpose(1, 0, 2)).max()
        assert err < KERNEL_BOUND, (r, err)


# ----------------------------------------------------------------------------- cfg 4
@pytest.mark.gpu
def test_cfg4_encode_of_16384_tokens():
    """(i) Given the oracle's fp32 inputs (its SVD cores, its residual R, V), the kernels write the
    oracle's slot bytes exactly. (ii) End to end from raw K (this repository's device fit, both
    decompositions), the per-field mismatch rates against the oracle's own encode."""
    from vllm_ttkv import encode, ops
    from vllm_ttkv.layout import config
    n = 16384
    g = O.geometry_for_config("tight", 110)
    lay = _lay(g)
    K, V = S.synth_kv(40, n)
    K, V = S.round_to_dtype(K, "bfloat16"), S.round_to_dtype(V, "bfloat16")
    cores, _ = O.tt_svd(np.ascontiguousarray(K.transpose(1, 2, 0)), 0.20, g.r1)
    f = O.fit_into_budget(K, g, "tight", "recip", cores=cores)
    want = O.build_slots(g, f["coeff_q"], f["coeff_scale"], f["R"], V, "recip")
    # (i)
    ft = ops.fit_tail(torch.from_numpy(cores[0][0]).cuda(), torch.from_numpy(cores[1]).cuda(),
                      torch.from_numpy(cores[2][:, :, 0]).cuda(), g.r1)
    assert np.array_equal(ft["coeff_q"].cpu().numpy(), f["coeff_q"])
    assert np.array_equal(ft["coeff_scale"].half().cpu().numpy().view(np.uint16),
                          f["coeff_scale"].view(np.uint16))
    assert np.array_equal(ft["dec_q"].cpu().numpy(), f["dec_q"])
    fk = encode.FittedK(ft["coeff_q"], ft["coeff_scale"], encode.KDecoder(ft["decoder"]), ft["dec_q"],
                        ft["dec_scale"], f["fitted_rank"], g.r1)
    Kd = torch.from_numpy(K).cuda().bfloat16().permute(1, 0, 2).contiguous()
    Vd = torch.from_numpy(V).cuda().bfloat16().permute(1, 0, 2).contiguous()
    slots = torch.arange(n, device="cuda")
    cache = torch.zeros(n, g.blob_bytes, dtype=torch.uint8, device="cuda")
    encode.write_fitted(cache, slots, fk, Kd, Vd, lay)
    ops.reset_status()
    ops.select_pack_rows(cache, slots, torch.from_numpy(f["R"]).cuda(), field_off=g.coeff_bytes + 2,
                         row_stride=g.k_row_bytes, lanes=g.res_k, bits=g.res_bits, heads=g.H, d=g.d)
    ops.check_status()
    assert np.array_equal(cache.cpu().numpy(), want), "slot bytes given the oracle's inputs"
    # (ii)
    ks_w = want[:, :g.k_slot_bytes]
    dense_want = O.dense_k(g, ks_w, f["decoder_f"])
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))   # noqa: E731
    cb = g.coeff_bytes + 2
    for method in ("gram", "svd"):
        G1, G2, G3 = encode.tt_svd_cores(torch.from_numpy(K).cuda(), 0.20, g.r1, method=method)
        out = ops.fit_tail(G1, G2, G3, g.r1)
        fk = encode.FittedK(out["coeff_q"], out["coeff_scale"], encode.KDecoder(out["decoder"]),
                            out["dec_q"], out["dec_scale"], int(G1.shape[1]), g.r1)
        cache.zero_()
        encode.write_fitted(cache, slots, fk, Kd, Vd, lay)
        got = cache.cpu().numpy()
        ks = got[:, :g.k_slot_bytes]
        dense_got = O.dense_k(g, ks, out["decoder"].cpu().numpy())
        rates = {"V bytes": float((got[:, g.k_slot_bytes:] != want[:, g.k_slot_bytes:]).mean()),
                 "coefficient block": float((ks[:, :cb] != ks_w[:, :cb]).mean()),
                 "K residual fields": float((ks[:, cb:] != ks_w[:, cb:]).mean()),
                 "decoded K vs oracle's (rel)": rel(dense_got, dense_want),
                 "decoded K vs raw K (rel), ours / oracle's": (rel(dense_got, K), rel(dense_want, K))}
        print(f"cfg4 end-to-end mismatch rates ({method}):", rates)
        assert rates["V bytes"] == 0.0
        assert rel(dense_got, K) <= 1.01 * rel(dense_want, K) + 1e-4     # reconstruction as good
        # two valid encodings of the same keys (the decompositions agree up to the order, sign and
        # rotation of near-equal singular directions, so codes move where a value sits near a
        # rounding boundary): the decoded keys agree to a few percent of |K|, the quantisation
        # noise level, and each reconstructs K as well as the other (above)
        assert rates["decoded K vs oracle's (rel)"] < 5e-2
