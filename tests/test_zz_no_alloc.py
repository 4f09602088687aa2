"""The allocation-free decode entry point, `ttkv_decode_paged_noalloc`, called through the C ABI.

It exists for callers that cannot hand the library scratch memory: hosts that reach the kernels
only through the C ABI with no device allocator of their own, and engines that fix their device
memory budget up front (vLLM sizes its KV cache from what a profiling pass leaves free, so memory
taken outside its pool mid-serving can push a later allocation out of memory). Its split-K
partials live in a static device array of TTKV_NOALLOC_SCRATCH_BYTES (4 MiB) per GPU instead of a
caller workspace.

Checked here: two calls in a row (two different stores, so the second call runs over the first
call's leftover scratch) agree with `ttkv_decode_paged` + workspace within the read-path
tolerance, and a decode needing more scratch than the array holds is refused before any launch.
The file is named to be collected last, so a run that stops at the first failure has already run
every other test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import stores
from vllm_ttkv import _lib, ops
from vllm_ttkv.layout import TTKLayout

pytestmark = pytest.mark.gpu

ATOL = 2e-3          # the read-path tolerance on attention outputs (fp16 store)


def _device_store(st):
    g = st["g"]
    lay = TTKLayout(H=g.H, d=g.d, r1=g.r1, qbits=g.qbits, res_k=g.res_k, res_bits=g.res_bits,
                    v_lanes=g.v_lanes, v_bits=g.v_bits)
    dev = "cuda"
    return dict(lay=lay, cache=torch.from_numpy(st["cache"]).to(dev),
                bt=torch.from_numpy(st["block_table"]).to(dev),
                seq=torch.from_numpy(st["seq_lens"]).to(dev),
                dec=torch.from_numpy(st["decoders"]).to(dev),
                idx=torch.arange(len(st["seq_lens"]), dtype=torch.int32, device=dev),
                table=torch.from_numpy(st["table"]).to(dev).half(),
                q=torch.from_numpy(st["q"]).to(dev).half())


def _noalloc(d, out, max_seq, status):
    """One call of ttkv_decode_paged_noalloc with plain pointers (no workspace argument)."""
    lib = _lib.lib()
    la = d["lay"].abi()
    cache = _lib.Cache(d["cache"].data_ptr(), d["cache"].shape[0], d["cache"].stride(0), 16, 0)
    batch = _lib.Batch(d["bt"].data_ptr(), d["bt"].stride(0), d["bt"].shape[1], d["seq"].data_ptr(),
                       d["bt"].shape[0], d["dec"].data_ptr(), d["dec"].stride(0), d["idx"].data_ptr(),
                       d["dec"].shape[0])
    rope = _lib.Rope(d["table"].data_ptr(), _lib.F16, d["table"].shape[0])
    HQ = d["q"].shape[1]
    return lib.ttkv_decode_paged_noalloc(
        C.byref(la), C.byref(cache), C.byref(batch), C.byref(rope), d["q"].data_ptr(), _lib.F16,
        HQ * 128, HQ, 128 ** -0.5, 0, d["lay"].H, out.data_ptr(), _lib.F32, HQ * 128, max_seq,
        status.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row():
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for seed, lens, cfg, r1 in ((21, [70, 33, 129], "safe", 32), (22, [300, 5], "tight", 48)):
        st = stores.make_store(seed, lens, cfg=cfg, r1=r1)
        d = _device_store(st)
        B, HQ = d["q"].shape[:2]
        max_seq = int(st["seq_lens"].max())
        want = torch.zeros(B, HQ, 128, device="cuda")
        ops.decode_paged(d["lay"], d["cache"], 16, d["bt"], d["seq"], d["dec"], d["idx"], d["table"],
                         d["q"], 128 ** -0.5, want, max_seq, status=status)
        got = torch.full((B, HQ, 128), float("nan"), device="cuda")
        assert _noalloc(d, got, max_seq, status) == _lib.OK, _lib.lib().ttkv_last_error()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        err = (got - want).abs().max().item()
        assert err < ATOL, (seed, err)
        assert np.abs(got.cpu().numpy() - stores.expected_decode(st)).max() < ATOL


def test_noalloc_refuses_a_decode_larger_than_its_scratch():
    st = stores.make_store(23, [40], cfg="safe", r1=32)
    d = _device_store(st)
    n = 2048                                   # 2048 requests x 24 query heads of partials > 4 MiB
    d["bt"] = d["bt"][:1].expand(n, -1).contiguous()
    d["seq"] = d["seq"][:1].expand(n).contiguous()
    d["idx"] = torch.zeros(n, dtype=torch.int32, device="cuda")
    d["q"] = d["q"][:1].expand(n, -1, -1).contiguous()
    la = d["lay"].abi()
    need = _lib.lib().ttkv_decode_workspace_bytes(C.byref(la), n, 24, 40, 0, 8)
    assert need > _lib.NOALLOC_SCRATCH_BYTES
    out = torch.zeros(n, 24, 128, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _noalloc(d, out, 40, status) == _lib.ERR_WORKSPACE
    assert b"TTKV_NOALLOC_SCRATCH_BYTES" in _lib.lib().ttkv_last_error()
    torch.cuda.synchronize()
    assert not out.any(), "a refused call must not launch"
