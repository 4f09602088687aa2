"""TT-KV compressed-KV attention for vLLM, on hand-written sm_100a CUDA (B200).

The package keeps the reference plugin's module surface (layout, decode, encode, impl,
metadata, rope_store) and routes every hot-path op through `libttkv_sm100.so` (see `ops`).
"""
__all__ = ["layout", "ops", "synthetic"]
