"""Generate the golden vectors that pin the oracle to the reference implementation.

Run once, in a container that has the reference's source tree (a path is given on the command
line; nothing at test time reads it):

    python tests/golden/make_golden.py /path/to/ttkv-vllm

It imports the reference's own Python modules (codec/ttkv_packed_cache.py, codec/ttkv_codec.py,
vllm_ttkv/{layout,reference,decode,encode}.py), feeds them seeded inputs on the CPU and stores
inputs + outputs as small `.npz` files beside this script, plus `manifest.json` with a SHA-256 of
every reference file used.

Two arithmetic modes, because the reference's format has two spellings of one rule
(`tensor / python_int` is a true division on CPU and a multiply by the fp32 reciprocal on CUDA,
vllm_ttkv/select_triton.py:76-84):
  * "true"  -- the reference exactly as it runs on a CPU;
  * "recip" -- the same code with `float32_tensor / python_number` routed through
    `tensor * float32(1/number)`, which is what ATen's CUDA true-divide kernel does for a CPU
    scalar divisor. This is the serving path's arithmetic and the one the CUDA kernels match.
"""
from __future__ import annotations

import contextlib
import hashlib
import importlib.util
import json
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parents[1]


def _load_synthetic():
    spec = importlib.util.spec_from_file_location(
        "ttkv_synthetic", REPO / "ttkv-vllm_b200" / "vllm_ttkv" / "synthetic.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _tie_free_rows(rng, rows, k, cast):
    """[rows, 128] fp32 whose k-th and (k+1)-th largest magnitudes differ in every row, so the
    kept lane SET is unique (torch.topk leaves the order of equal magnitudes unspecified)."""
    out = []
    while len(out) < rows:
        x = cast(rng.standard_normal(128).astype(np.float32))
        m = np.sort(np.abs(x))[::-1]
        if k >= 128 or m[k - 1] != m[k]:
            out.append(x)
    return np.stack(out).astype(np.float32)


def _untie_v(rng, V, k, syn):
    """Redraw the (head, token) rows of an fp16-rounded V whose k-th and (k+1)-th magnitudes
    tie, so the V lane selection is unique (see `_tie_free_rows`)."""
    H, n, d = V.shape
    rows = V.reshape(H * n, d).copy()
    for i in range(rows.shape[0]):
        while True:
            m = np.sort(np.abs(rows[i]))[::-1]
            if m[k - 1] != m[k]:
                break
            rows[i] = syn.round_to_dtype(rng.standard_normal(d).astype(np.float32), "float16")
    return rows.reshape(H, n, d)


@contextlib.contextmanager
def cuda_division_rule(torch):
    """Route fp32 `tensor / python_number` through a multiply by the fp32 reciprocal."""
    orig = torch.Tensor.__truediv__

    def div(self, other):
        if isinstance(other, (int, float)) and not isinstance(other, bool) \
                and self.dtype == torch.float32:
            inv = np.float32(1.0) / np.float32(other)
            return self * torch.tensor(inv, dtype=torch.float32)
        return orig(self, other)

    torch.Tensor.__truediv__ = div
    try:
        yield
    finally:
        torch.Tensor.__truediv__ = orig


def main(ref_root: str):
    ref = pathlib.Path(ref_root).resolve()
    sys.path.insert(0, str(ref / "codec"))
    sys.path.insert(0, str(ref))
    import torch
    import ttkv_codec as codec
    import ttkv_packed_cache as pc
    from vllm_ttkv import decode as dc
    from vllm_ttkv import encode as enc
    from vllm_ttkv import layout as L
    from vllm_ttkv import reference as R

    syn = _load_synthetic()
    torch.manual_seed(0)
    used = ["codec/ttkv_packed_cache.py", "codec/ttkv_codec.py", "vllm_ttkv/layout.py",
            "vllm_ttkv/reference.py", "vllm_ttkv/decode.py", "vllm_ttkv/encode.py"]
    manifest = {"reference_files": {f: hashlib.sha256((ref / f).read_bytes()).hexdigest()
                                    for f in used},
                "torch": torch.__version__, "numpy": np.__version__, "cases": {}}

    def save(name, **arrays):
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        manifest["cases"][name] = sorted(arrays)

    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))       # noqa: E731
    N = lambda t: t.detach().cpu().numpy()                          # noqa: E731

    # ---------------------------------------------------------------- A. geometry
    geo = []
    for cfg in ("safe", "tight", "campaign4x"):
        for r1 in (14, 24, 33, 61, 64, 110, 112, 143):
            lay = L.layout_for_config(codec.CONFIGS[cfg], r1)
            geo.append(dict(cfg=cfg, r1=r1, H=lay.H, d=lay.d, qbits=lay.qbits, res_k=lay.res_k,
                            res_bits=lay.res_bits, v_lanes=lay.v_lanes, v_bits=lay.v_bits,
                            coeff_bytes=lay.coeff_bytes, k_row_bytes=lay.k_row_bytes,
                            v_row_bytes=lay.v_row_bytes, k_slot_bytes=lay.k_slot_bytes,
                            v_slot_bytes=lay.v_slot_bytes, v_offset=lay.v_offset,
                            blob_bytes=lay.compressed_bytes_per_token()))
    (HERE / "geometry.json").write_text(json.dumps(geo, indent=1))
    manifest["cases"]["geometry"] = ["json"]

    # ---------------------------------------------------------------- B. bit packing
    rng = np.random.default_rng(1)
    bits_cases = {}
    for k, bits in ((81, 3), (32, 3), (45, 3), (64, 4), (17, 2), (5, 8), (1, 3)):
        vals = rng.integers(0, 2 ** bits, size=(16, k))
        packed = N(pc.pack_bits_rows(T(vals), bits))
        back = N(pc.unpack_bits_rows(T(packed), k, bits))
        assert (back == vals).all()
        bits_cases[f"vals_{k}_{bits}"] = vals.astype(np.int32)
        bits_cases[f"packed_{k}_{bits}"] = packed
    bm = rng.integers(0, 256, size=(16, 16), dtype=np.uint8)
    bits_cases["bitmap_in"] = bm
    bits_cases["bitmap_out"] = N(pc.unpack_bitmap_rows(T(bm), 128))
    save("bits", **bits_cases)

    # ---------------------------------------------------------------- C. row containers
    for mode in ("true", "recip"):
        ctx = cuda_division_rule(torch) if mode == "recip" else contextlib.nullcontext()
        rows = {}
        with ctx:
            for k, bits in ((81, 3), (32, 3), (45, 3), (64, 4)):
                for kind in ("f32", "bf16"):
                    X = _tie_free_rows(rng, 16, k, (lambda a: syn.round_to_dtype(a * 3, "bfloat16"))
                                       if kind == "bf16" else (lambda a: a))
                    Xt = T(X)
                    mask = pc._topk_mask(Xt, k)
                    pr = pc.PackedRows.build(Xt, mask, bits, 128, k=k, check=False)
                    tag = f"{k}_{bits}_{kind}"
                    rows[f"X_{tag}"] = X
                    rows[f"bitmap_{tag}"] = N(pr.bitmap)
                    rows[f"packed_{tag}"] = N(pr.packed)
                    rows[f"scale_{tag}"] = N(pr.scale).view(np.uint16)
                    rows[f"dense_{tag}"] = N(pr.materialise(torch.float32))
                # all-zero rows: the ruler is 1/(2^(b-1)-1); the lane choice is a tie
                Z = torch.zeros(4, 128)
                pr = pc.PackedRows.build(Z, pc._topk_mask(Z, k), bits, 128, k=k, check=False)
                rows[f"zero_scale_{k}_{bits}"] = N(pr.scale).view(np.uint16)
                rows[f"zero_dense_{k}_{bits}"] = N(pr.materialise(torch.float32))
            M = rng.standard_normal((24, 1024)).astype(np.float32)
            M[3] = 0.0
            q, s = pc._quant_rows(T(M), 8)
            rows["qr_in"], rows["qr_q"], rows["qr_s"] = M, N(q), N(s).view(np.uint16)
        save(f"rows_{mode}", **rows)

    # ---------------------------------------------------------------- D/E/F. fit, encode, read
    for mode, cfgname, n, budget, seed in (("true", "safe", 48, 24, 3), ("recip", "safe", 48, 24, 3),
                                           ("recip", "campaign4x", 40, 16, 5),
                                           ("recip", "tight", 36, 20, 7)):
        cfg = codec.CONFIGS[cfgname]
        lay = L.layout_for_config(cfg, budget)
        K, V = syn.synth_kv(seed, n + 5)
        K = syn.round_to_dtype(K, "float16")        # stored compactly, exact as fp32
        V = _untie_v(rng, syn.round_to_dtype(V, "float16"), cfg["k_lanes"], syn)
        Kp, Kn = K[:, :n], K[:, n:]
        Vp, Vn = V[:, :n], V[:, n:]
        out = {"K": K.astype(np.float16), "V": V.astype(np.float16)}
        ctx = cuda_division_rule(torch) if mode == "recip" else contextlib.nullcontext()
        with ctx:
            Xt = T(np.ascontiguousarray(Kp.transpose(1, 2, 0)))
            cores, ranks = codec.tt_svd(Xt, cfg["tols"], budget)
            fk = enc.fit_into_budget(T(Kp), lay, cfg)
            out.update(G1=N(cores[0]), G2=N(cores[1]), G3=N(cores[2]),
                       fit_coeff_q=N(fk.coeff_q), fit_coeff_scale=N(fk.coeff_scale).view(np.uint16),
                       fit_rank=np.int32(fk.fitted_rank))
            kl = pc.build_k_layer(T(Kp), cfg["tols"], cfg["qbits"], cfg["res_frac"],
                                  cfg["res_bits"], max_rank=budget)
            out.update(fit_dec_q=N(kl.dec_q), fit_dec_scale=N(kl.dec_scale).view(np.uint16),
                       fit_res_bitmap=N(kl.resid.bitmap), fit_res_packed=N(kl.resid.packed),
                       fit_res_scale=N(kl.resid.scale).view(np.uint16))
            vrows = enc.encode_v(T(Vp), lay)
            ks = L.pack_k_slots(lay, fk.coeff_q, fk.coeff_scale, fk.resid)
            vs = L.pack_v_slots(lay, vrows)
            out.update(k_slots=N(ks), v_slots=N(vs))
            # frozen projection of the 5 later tokens against the fitted decoder
            kdec = fk.decoder
            fz = enc.encode_frozen(T(np.ascontiguousarray(Kn)), kdec, lay)
            out.update(pinv=N(kdec.pinv), fz_coeff_q=N(fz.coeff_q),
                       fz_coeff_scale=N(fz.coeff_scale).view(np.uint16), fz_R=N(fz.resid_src))
            zks = L.pack_k_slots(lay, fz.coeff_q, fz.coeff_scale, fz.resid)
            zvs = L.pack_v_slots(lay, enc.encode_v(T(np.ascontiguousarray(Vn)), lay))
            out.update(fz_k_slots=N(zks), fz_v_slots=N(zvs))
            # the read, over all n + 5 stored rows
            ks_all = torch.cat([ks, zks])
            vs_all = torch.cat([vs, zvs])
            m = n + 5
            table = syn.cos_sin_cache(m + 3, dtype="float16")
            cos, sin = dc.cos_sin_from_cache(T(table).half(), torch.arange(m), 128)
            q = syn.synth_queries(seed, (24, 128), "float16")
            dec = kdec.decoder_f
            out.update(table=table.astype(np.float16), q=q.astype(np.float16),
                       dense_k=N(R.dense_k_from_slots(lay, ks_all, dec))[:, :4],
                       dense_v=N(R.dense_v_from_slots(lay, vs_all))[:, :4],
                       scores=N(R.raw_scores(lay, ks_all, dec, T(q), cos, sin)),
                       attend=N(R.attend_raw_store(lay, ks_all, vs_all, dec, T(q), cos, sin)),
                       attend_oracle=N(R.oracle_attend(lay, ks_all, vs_all, dec, T(q), cos, sin)))
            Q = 6
            qm = syn.synth_queries(seed + 1, (24, Q, 128), "float16")
            p0 = m - Q
            sm = R.raw_scores_multi(lay, ks_all, dec, T(qm), cos, sin, p0=p0)
            p = torch.softmax(sm, dim=-1)
            Vd = R.dense_v_from_slots(lay, vs_all)
            p_all = torch.arange(24) // 3
            om = torch.einsum("hqn,hnd->hqd", p, Vd[p_all])
            out.update(qm=qm.astype(np.float16), p0=np.int32(p0), scores_multi=N(sm),
                       attend_multi=N(om))
        save(f"store_{cfgname}_{mode}", **out)

    # ---------------------------------------------------------------- G. paging
    bt, total = syn.block_table(11, [37, 5, 64, 1], 16)
    slots = [N(dc.block_slots(T(bt[r]), n, 16)) for r, n in enumerate([37, 5, 64, 1])]
    save("paging", block_table=bt, seq_lens=np.array([37, 5, 64, 1], np.int32),
         slots=np.concatenate(slots))

    cfg0(torch, codec, pc, dc, enc, L, R, syn, save, manifest)
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1))
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


CFG0_N, CFG0_R1 = 1082, 110


def cfg0(torch, codec, pc, dc, enc, L, R, syn, save, manifest):
    """H. BASELINE config 0 at its full size: one request of 1082 tokens, r1 = 110, `safe`, an fp16
    model (K, V, q and the llama3-scaled RoPE table in fp16), encoded by the reference's own
    encoder (fit_into_budget + pack_{k,v}_slots) and read by its CPU path (attend_raw_store).
    K and V are not stored: they are `synth_kv(seed, 1082)` rounded to fp16 (checked by SHA-256),
    except the (head, token) rows of V whose 81st and 82nd largest magnitudes tie (about 1% of
    fp16 rows), which are redrawn so that the reference's torch.topk lane set is unique; those
    rows are stored (`v_fix_rows`, `v_fix`)."""
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))       # noqa: E731
    N = lambda t: t.detach().cpu().numpy()                          # noqa: E731
    cfg = codec.CONFIGS["safe"]
    lay = L.layout_for_config(cfg, CFG0_R1)
    seed = 100
    K, V0 = syn.synth_kv(seed, CFG0_N)
    K = syn.round_to_dtype(K, "float16")
    V0 = syn.round_to_dtype(V0, "float16")
    V = _untie_v(np.random.default_rng(seed + 1), V0, cfg["k_lanes"], syn)
    fix = np.nonzero(np.any(V.reshape(-1, 128) != V0.reshape(-1, 128), axis=1))[0].astype(np.int32)
    out = {"seed": np.int32(seed), "n": np.int32(CFG0_N), "r1": np.int32(CFG0_R1),
           "v_fix_rows": fix, "v_fix": V.reshape(-1, 128)[fix].astype(np.float16),
           "K_sha256": np.frombuffer(hashlib.sha256(K.astype(np.float16).tobytes()).digest(), np.uint8),
           "V_sha256": np.frombuffer(hashlib.sha256(V0.astype(np.float16).tobytes()).digest(), np.uint8)}
    with cuda_division_rule(torch):
        Xt = T(np.ascontiguousarray(K.transpose(1, 2, 0)))
        cores, _ = codec.tt_svd(Xt, cfg["tols"], CFG0_R1)
        fk = enc.fit_into_budget(T(K), lay, cfg)
        kl = pc.build_k_layer(T(K), cfg["tols"], cfg["qbits"], cfg["res_frac"], cfg["res_bits"],
                              max_rank=CFG0_R1)
        dec = fk.decoder.decoder_f
        r = int(fk.fitted_rank)
        dq, ds = N(kl.dec_q), N(kl.dec_scale)
        assert np.array_equal(N(dec)[:r], dq.astype(np.float32) * ds.astype(np.float32)[:, None])
        ks = L.pack_k_slots(lay, fk.coeff_q, fk.coeff_scale, fk.resid)
        vs = L.pack_v_slots(lay, enc.encode_v(T(V), lay))
        table = syn.cos_sin_cache(CFG0_N + 6, dtype="float16")
        cos, sin = dc.cos_sin_from_cache(T(table).half(), torch.arange(CFG0_N), 128)
        q = syn.synth_queries(seed, (24, 128), "float16")
        out.update(G1=N(cores[0]), G2=N(cores[1]), G3=N(cores[2]), fit_rank=np.int32(r),
                   dec_q=dq, dec_scale=ds.view(np.uint16), k_slots=N(ks), v_slots=N(vs),
                   q=q.astype(np.float16),
                   attend=N(R.attend_raw_store(lay, ks, vs, dec, T(q), cos, sin)),
                   attend_oracle=N(R.oracle_attend(lay, ks, vs, dec, T(q), cos, sin)))
    save("store_cfg0_recip", **out)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    if len(args) != 1:
        sys.exit("usage: make_golden.py <reference source tree> [--only-cfg0]")
    if "--only-cfg0" in sys.argv:
        # add config 0's case to an existing golden set (the other files are left as they are)
        ref = pathlib.Path(args[0]).resolve()
        sys.path.insert(0, str(ref / "codec"))
        sys.path.insert(0, str(ref))
        import torch
        import ttkv_codec as codec
        import ttkv_packed_cache as pc
        from vllm_ttkv import decode as dc
        from vllm_ttkv import encode as enc
        from vllm_ttkv import layout as L
        from vllm_ttkv import reference as R
        manifest = json.loads((HERE / "manifest.json").read_text())

        def save(name, **arrays):
            np.savez_compressed(HERE / f"{name}.npz", **arrays)
            manifest["cases"][name] = sorted(arrays)
        cfg0(torch, codec, pc, dc, enc, L, R, _load_synthetic(), save, manifest)
        (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1))
        print("wrote store_cfg0_recip.npz")
    else:
        main(args[0])
