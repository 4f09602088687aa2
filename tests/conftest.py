"""Shared test setup: import paths and the `gpu` marker.

`-m "not gpu"` runs the oracle-vs-golden pins, the host logic and the C-ABI symbol checks on a CPU;
`-m gpu` runs the parity tests proper, through the C ABI, on a B200.
"""
import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "ttkv-vllm_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
