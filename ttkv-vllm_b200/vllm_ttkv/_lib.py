"""ctypes binding of `libttkv_sm100.so` (the C ABI declared in `include/ttkv_b200.h`).

The library is built in-tree (`vllm_ttkv._build.build()`, or `__graft_entry__.build()`) and loaded
from the package directory. There is no fallback: if the library is missing or was built for a
different ABI version, `lib()` raises, and so does every op that needs it.
"""
from __future__ import annotations

import ctypes as C
import pathlib

ABI_VERSION = 5
LIB_PATH = pathlib.Path(__file__).resolve().parents[1] / "libttkv_sm100.so"

# host-side refusal codes (ttkv_b200.h)
OK = 0
ERR_ARG, ERR_LAYOUT, ERR_UNSUPPORTED, ERR_ALIGN, ERR_WORKSPACE, ERR_CUDA = -1, -2, -3, -4, -5, -6
# device status codes
STATUS = {0: "ok", 1: "block index outside the cache", 2: "block-table row too short for seq_len",
          3: "decoder index outside the pool", 4: "slot id is PAD_SLOT_ID or outside the cache",
          5: "query range inconsistent with seq_len",
          6: "a bounded wait on the tensor-core pipeline ran out",
          7: "a seq_len above the max_seq_len the read was given (its bound)"}

F32, F16, BF16 = 0, 1, 2
CACHE_SKIP_PAD = 1                          # TTKV_CACHE_SKIP_PAD
NOALLOC_SCRATCH_BYTES = 4 * 1024 * 1024   # TTKV_NOALLOC_SCRATCH_BYTES


class Layout(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "H", "d", "r1", "qbits", "res_k", "res_bits", "v_lanes", "v_bits", "align",
        "coeff_bytes", "k_row_bytes", "v_row_bytes", "k_slot_bytes", "v_slot_bytes", "v_offset",
        "blob_bytes")]


class Cache(C.Structure):
    _fields_ = [("base", C.c_void_p), ("n_slots", C.c_int64), ("row_bytes", C.c_int64),
                ("block_size", C.c_int32), ("flags", C.c_int32)]


class Batch(C.Structure):
    _fields_ = [("block_table", C.c_void_p), ("bt_stride", C.c_int64), ("bt_cols", C.c_int32),
                ("seq_lens", C.c_void_p), ("n_reqs", C.c_int32), ("decoders", C.c_void_p),
                ("dec_stride", C.c_int64), ("dec_index", C.c_void_p), ("n_decoders", C.c_int32),
                ("dec_image", C.c_void_p), ("image_stride", C.c_int64), ("dec_scales", C.c_void_p)]


class Rope(C.Structure):
    _fields_ = [("table", C.c_void_p), ("dtype", C.c_int32), ("rows", C.c_int64)]


MAX_PEERS = 8                               # TTKV_MAX_PEERS


class Peers(C.Structure):
    """ttkv_peers_t: the group of a gathered decode (every rank's output and signal word as mapped
    in this process, and this rank's epoch word)."""
    _fields_ = [("world", C.c_int32), ("rank", C.c_int32), ("out", C.c_void_p * MAX_PEERS),
                ("signal", C.c_void_p * MAX_PEERS), ("epoch", C.c_void_p), ("ticket", C.c_void_p)]


P, I32, I64, SZ, F = C.c_void_p, C.c_int32, C.c_int64, C.c_size_t, C.c_float
LP, CP, BP, RP = C.POINTER(Layout), C.POINTER(Cache), C.POINTER(Batch), C.POINTER(Rope)
PP = C.POINTER(Peers)

# name -> (restype, argtypes); every symbol the header declares
SIGNATURES = {
    "ttkv_layout_init": (C.c_int, [LP, I32, I32, I32, I32, I32, I32, I32, I32, I32]),
    "ttkv_last_error": (C.c_char_p, []),
    "ttkv_abi_version": (I32, []),
    "ttkv_decode_workspace_bytes": (SZ, [LP, I32, I32, I32, I32, I32]),
    "ttkv_decoder_image_bytes": (SZ, [LP]),
    "ttkv_decoder_image": (C.c_int, [LP, P, I64, I32, P, I64, P, P]),
    "ttkv_decode_paged": (C.c_int, [LP, CP, BP, RP, P, I32, I64, I32, F, I32, I32, P, I32, I64,
                                    I32, P, SZ, P, P]),
    "ttkv_decode_paged_noalloc": (C.c_int, [LP, CP, BP, RP, P, I32, I64, I32, F, I32, I32, P,
                                            I32, I64, I32, P, P]),
    "ttkv_decode_paged_gather": (C.c_int, [LP, CP, BP, RP, P, I32, I64, I32, F, I32, I32, P, I32,
                                           I64, I32, P, SZ, PP, P, P]),
    "ttkv_peer_wait": (C.c_int, [PP, I64, P, P]),
    "ttkv_ipc_handle_bytes": (SZ, []),
    "ttkv_ipc_alloc": (C.c_int, [SZ, C.POINTER(C.c_void_p), P]),
    "ttkv_ipc_open": (C.c_int, [P, C.POINTER(C.c_void_p)]),
    "ttkv_ipc_close": (C.c_int, [P]),
    "ttkv_ipc_free": (C.c_int, [P]),
    "ttkv_prefill_workspace_bytes": (SZ, [LP, I32, I32, I32, I32, I32, I32]),
    "ttkv_prefill_cont_paged": (C.c_int, [LP, CP, BP, RP, P, P, P, I32, I64, I32, F, I32, I32,
                                          P, I32, I64, I32, I32, P, SZ, P, P]),
    "ttkv_write_workspace_bytes": (SZ, [LP, I32]),
    "ttkv_write_paged": (C.c_int, [LP, CP, P, I32, P, I32, I64, P, I32, I64, P, P, I64, P, I64,
                                   I32, P, P, P, SZ, P, P]),
    "ttkv_write_paged_shard": (C.c_int, [LP, I32, I32, CP, P, I32, P, I32, I64, P, I32, I64, P, P,
                                         I64, P, I64, I32, P, P, P, SZ, P, P]),
    "ttkv_select_pack_rows": (C.c_int, [CP, P, I32, P, I32, I32, I32, I32, I32, I32, I32, P, P]),
    "ttkv_fit_tail_scratch_bytes": (SZ, [I32, I32, I32, I32]),
    "ttkv_fit_tail": (C.c_int, [P, P, P, I32, I32, I32, I32, I32, I32, I32, P, P, P, P, P, P, SZ,
                                P]),
}

_LIB = None


class TTKVError(RuntimeError):
    """A refusal returned by the C ABI (message from `ttkv_last_error`)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"ttkv error {code}: {msg}")
        self.code = code


def load(path=LIB_PATH):
    """Load the shared library and bind every declared symbol; raise if anything is missing."""
    if not pathlib.Path(path).exists():
        raise ImportError(
            f"{path} is missing: the TT-KV CUDA library has not been built. Run "
            f"`python -c 'import __graft_entry__; __graft_entry__.build()'` (or "
            f"`vllm_ttkv._build.build()`). There is no CPU or Triton fallback.")
    lib = C.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)                      # AttributeError if not exported
        fn.restype, fn.argtypes = res, args
    if lib.ttkv_abi_version() != ABI_VERSION:
        raise ImportError(f"{path} has ABI version {lib.ttkv_abi_version()}, expected {ABI_VERSION}")
    return lib


def lib():
    global _LIB
    if _LIB is None:
        _LIB = load()
    return _LIB


def check(code: int):
    if code != OK:
        raise TTKVError(code, lib().ttkv_last_error().decode(errors="replace"))


def check_with(library, code: int):
    """`check` against a given library object (the loaded one, or a stand-in in tests)."""
    if code != OK:
        raise TTKVError(code, library.ttkv_last_error().decode(errors="replace"))
