"""The TT-SVD fit's decompositions on the CPU (torch): the Gram-matrix route gives the SVD's rank
and reconstruction, which is how this build defines parity for a faster fit (the reference's own
tests pin no singular vectors, only self-consistency of the fit)."""
import numpy as np
import pytest
import torch

from vllm_ttkv import encode
from vllm_ttkv import synthetic as S


def _recon(G1, G2, G3):
    r, d, r2 = G2.shape
    return G1 @ torch.einsum("rdq,qh->rdh", G2, G3).reshape(r, -1)


@pytest.mark.parametrize("n,cap", [(3000, 110), (5000, 143), (2100, 14), (1082, 110), (600, 110),
                                   (256, 67)])
def test_gram_fit_matches_the_svd_fit(n, cap):
    K = torch.from_numpy(S.synth_kv(7, n)[0])
    H, _, d = K.shape
    X = K.permute(1, 2, 0).reshape(n, d * H)
    cores = {m: encode.tt_svd_cores(K, 0.2, cap, m) for m in ("svd", "gram")}
    (a1, a2, a3), (b1, b2, b3) = cores["svd"], cores["gram"]
    assert a1.shape == b1.shape and a2.shape == b2.shape and a3.shape == b3.shape   # the ranks
    ea = float((X - _recon(*cores["svd"])).norm() / X.norm())
    eb = float((X - _recon(*cores["gram"])).norm() / X.norm())
    assert abs(ea - eb) <= 1e-4 * max(ea, 1e-3), (ea, eb)
    # G1's columns are orthonormal in both
    for G1 in (a1, b1):
        np.testing.assert_allclose((G1.T @ G1).numpy(), np.eye(G1.shape[1]), atol=1e-3)


def test_gram_fit_of_low_rank_and_zero_keys():
    """A key block of rank 5 (the energy rule stops early) and an all-zero block (no NaN)."""
    rng = np.random.default_rng(0)
    low = rng.standard_normal((3000, 5)) @ rng.standard_normal((5, 1024))
    K = torch.from_numpy(low.astype(np.float32)).reshape(3000, 128, 8).permute(2, 0, 1).contiguous()
    G1, G2, G3 = encode.tt_svd_cores(K, 0.2, 110, "gram")
    # the energy rule keeps one direction past the last that it needs (the reference's count)
    assert G1.shape[1] == encode.tt_svd_cores(K, 0.2, 110, "svd")[0].shape[1] == 6
    X = K.permute(1, 2, 0).reshape(3000, 1024)
    assert float((X - _recon(G1, G2, G3)).norm() / X.norm()) <= 0.2
    Z = torch.zeros(8, 3000, 128)
    cores = encode.tt_svd_cores(Z, 0.2, 110, "gram")
    assert all(torch.isfinite(c).all() for c in cores)
    assert float(_recon(*cores).abs().max()) == 0.0


def test_fit_method_selection(monkeypatch):
    monkeypatch.delenv(encode.FIT_ENV, raising=False)
    assert encode.fit_method(4096, 1024) == "gram" and encode.fit_method(1082, 1024) == "gram"
    assert encode.fit_method(encode.GRAM_MIN_TOKENS - 1, 1024) == "svd"
    monkeypatch.setenv(encode.FIT_ENV, "svd")
    assert encode.fit_method(16384, 1024) == "svd"
    monkeypatch.setenv(encode.FIT_ENV, "bogus")
    with pytest.raises(ValueError):
        encode.fit_method(16384, 1024)
