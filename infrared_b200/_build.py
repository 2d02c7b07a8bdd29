"""Build ``libinfrared_b200.so`` in-tree with nvcc for sm_100a.

The library is plain CUDA C++ behind a C ABI (no torch headers), compiled
with ``-gencode arch=compute_100a,code=sm_100a`` and the static CUDA runtime,
so it loads next to any PyTorch build. ``python -m infrared_b200._build``
rebuilds it; ``build()`` skips the compile when the library is newer than
every source file.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libinfrared_b200.so"

SOURCES = ["capi.cu", "cache_ops.cu", "decode_generic.cu", "decode_tma.cu", "prefill_tc.cu",
           "peer_exchange.cu", "kv_proj.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; set NVCC or put CUDA's bin on PATH")
    return cand


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES]
    files += sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h"))
    files += sorted(INCLUDE.glob("*.h"))
    return files


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(f.stat().st_mtime <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False, out: Path | None = None,
          defines: tuple[str, ...] = ()) -> Path:
    """Compile the library (to ``out`` with extra ``-D`` defines for tuning
    variants; the default build goes next to this file)."""
    dst = Path(out) if out is not None else LIB
    if out is None and not defines and not force and up_to_date():
        return LIB
    cmd = [
        nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo",
        "-Xcompiler", "-fPIC,-O3", "-shared", "-cudart", "static",
        "--expt-relaxed-constexpr", "-I", str(INCLUDE),
        *[f"-D{d}" for d in defines],
        "-o", str(dst) + ".tmp",
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True, cwd=str(CSRC))
    os.replace(str(dst) + ".tmp", dst)
    return dst


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
