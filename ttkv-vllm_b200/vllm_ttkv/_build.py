"""Build `libttkv_sm100.so` in-tree with nvcc for sm_100a (B200)."""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess

PKG = pathlib.Path(__file__).resolve().parents[1]          # the ttkv-vllm_b200 directory
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OUT = PKG / "libttkv_sm100.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted(CSRC.glob("*.cu"))


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    return all(p.stat().st_mtime <= t for p in deps)


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    """Compile every .cu under csrc/ into one shared library next to the package."""
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           f"-I{INCLUDE}", f"-I{CSRC}", "-o", str(OUT) + ".tmp", *map(str, sources())]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force=True, verbose=True))
