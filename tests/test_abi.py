"""The C-ABI library loads on a CPU-only host, exports every function `include/*.h` declares,
and its host-only entry points (layout construction, workspace sizing) agree with the reference.
No kernel is launched here."""
import ctypes
import json
import pathlib
import re

import pytest

from conftest import GOLDEN, ROOT
from vllm_ttkv import _lib

HEADER = ROOT / "include" / "ttkv_b200.h"


def _declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    names = set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(ttkv_\w+)\s*\(", text, flags=re.M))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared()
    assert len(declared) >= 12, declared
    for name in declared:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) <= set(declared)
    assert lib.ttkv_abi_version() == _lib.ABI_VERSION


def test_layout_init_matches_reference_geometry():
    from vllm_ttkv.layout import layout_for_config
    for row in json.loads((GOLDEN / "geometry.json").read_text()):
        lay = layout_for_config(row["cfg"], row["r1"])
        st = lay.abi()
        for k in ("coeff_bytes", "k_row_bytes", "v_row_bytes", "k_slot_bytes", "v_slot_bytes",
                  "v_offset", "blob_bytes"):
            assert getattr(st, k) == row[k], (row["cfg"], row["r1"], k)
        assert lay.compressed_bytes_per_token() == row["blob_bytes"]


def test_layout_init_refusals():
    lib = _lib.load()
    st = _lib.Layout()
    for args in ((8, 100, 32, 8, 81, 3, 81, 3, 16),     # d % 8
                 (8, 128, 32, 8, 129, 3, 81, 3, 16),    # res_k > d
                 (8, 128, 32, 8, 81, 3, 200, 3, 16),    # v_lanes > d
                 (8, 128, 33, 4, 81, 3, 81, 3, 16)):    # r1*qbits % 8
        assert lib.ttkv_layout_init(ctypes.byref(st), *args) == _lib.ERR_LAYOUT
        assert lib.ttkv_last_error()


def test_workspace_sizes_are_host_computable():
    from vllm_ttkv.layout import layout_for_config
    lib = _lib.load()
    la = layout_for_config("safe", 110).abi()
    a = lib.ttkv_decode_workspace_bytes(ctypes.byref(la), 8, 24, 4322, 0, 8)
    b = lib.ttkv_decode_workspace_bytes(ctypes.byref(la), 8, 24, 4322, 0, 4)
    assert a > 0 and b > 0
    assert lib.ttkv_write_workspace_bytes(ctypes.byref(la), 8) == 8 * 110 * 4
    assert lib.ttkv_prefill_workspace_bytes(ctypes.byref(la), 4, 24, 256, 7379, 0, 8) > 0


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(ImportError, match="no CPU or Triton fallback"):
        _lib.load(tmp_path / "libttkv_sm100.so")


def test_ctypes_structs_match_the_header_layout(tmp_path):
    """Every struct the ctypes binding declares has the C header's size and field offsets (a C
    program built from include/ttkv_b200.h prints them)."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"ttkv_layout_t": _lib.Layout, "ttkv_cache_t": _lib.Cache, "ttkv_batch_t": _lib.Batch,
               "ttkv_rope_t": _lib.Rope, "ttkv_peers_t": _lib.Peers}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "ttkv_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c99", f"-I{HEADER.parent}", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l.strip()}
    for cname, py in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)
