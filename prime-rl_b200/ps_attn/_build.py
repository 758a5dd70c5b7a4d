"""Build recipe for libps_attn.so (sm_100a only).

The library is compiled in-tree next to this file so that it travels with the
repository; ``python -m ps_attn._build`` (with ``prime-rl_b200`` on
``sys.path``) or ``__graft_entry__.build()`` runs it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR.parent / "csrc"
REPO = PKG_DIR.parent.parent
INCLUDE = REPO / "include"
LIB_PATH = PKG_DIR / "libps_attn.so"

SOURCES = ["ps_attn_api.cu", "kv_append.cu", "paged_decode.cu", "chunked_prefill.cu",
           "paged_decode_static.cu", "cascade_plan.cu", "rope_append.cu", "dcp.cu",
           "head_gather.cu"]
HEADERS = ["ps_common.cuh", "ps_launch.h", "tcgen05.cuh", "peer_sync.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libps_attn.so")


def _inputs():
    files = [CSRC / s for s in SOURCES if (CSRC / s).exists()]
    files += [CSRC / h for h in HEADERS if (CSRC / h).exists()]
    files.append(INCLUDE / "ps_attn.h")
    files.append(Path(__file__))
    return files


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(f.stat().st_mtime > t for f in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False,
          out: Path | None = None, defines: dict | None = None) -> Path:
    """Compile the library.  ``out``/``defines`` build a tuning variant
    (e.g. ``{"PS_DECODE_STAGES": 4}``) at another path without touching the
    in-tree library."""
    target = Path(out) if out is not None else LIB_PATH
    if out is None and not defines and not force and not needs_build():
        return LIB_PATH
    nvcc = nvcc_path()
    srcs = [str(CSRC / s) for s in SOURCES if (CSRC / s).exists()]
    tmp = target.with_suffix(".so.tmp")
    cmd = [
        nvcc, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC,-O3", "-shared", "-cudart", "static",
        f"-I{INCLUDE}", f"-I{CSRC}", "-o", str(tmp), *srcs,
    ]
    for k, v in (defines or {}).items():
        cmd.insert(1, f"-D{k}={v}")
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_verbose:
        print(res.stdout + res.stderr, file=sys.stderr)
    os.replace(tmp, target)
    return target


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_verbose="--ptxas" in sys.argv)
    print(LIB_PATH)
