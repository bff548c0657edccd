"""Build the sm_100a shared library ``libnie_b200.so`` in-tree with nvcc.

The library is plain C ABI (``include/nie_b200.h``) with the CUDA runtime
linked statically, so it depends only on the NVIDIA driver at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "libnie_b200.so"
INCLUDE_DIR = PKG_DIR.parent / "include"

SOURCES = (
    "nie_runtime.cu",
    "nie_meta.cu",
    "nie_attn_generic.cu",
    "nie_attn_decode.cu",
    "nie_attn_prefill.cu",
    "nie_fused.cu",
)

ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")
COMMON_FLAGS = (
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3",
)


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _compile(src: Path, obj: Path, extra: tuple[str, ...]) -> None:
    cmd = [
        _nvcc(),
        *ARCH_FLAGS,
        *COMMON_FLAGS,
        *extra,
        "-I",
        str(INCLUDE_DIR),
        "-c",
        str(src),
        "-o",
        str(obj),
    ]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")


def _stale(force: bool) -> bool:
    if force or not LIB_PATH.exists():
        return True
    lib_time = LIB_PATH.stat().st_mtime
    inputs = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE_DIR.glob("*.h"))
    return any(p.stat().st_mtime > lib_time for p in inputs)


def build(force: bool = False, verbose: bool = False, extra_flags: tuple[str, ...] = ()) -> Path:
    """Compile every kernel source for sm_100a and link ``libnie_b200.so``."""
    if not _stale(force):
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    objs = [BUILD_DIR / (Path(s).stem + ".o") for s in SOURCES]
    with ThreadPoolExecutor(max_workers=min(8, len(SOURCES))) as pool:
        futures = [
            pool.submit(_compile, CSRC / s, o, tuple(extra_flags)) for s, o in zip(SOURCES, objs)
        ]
        for f in futures:
            f.result()
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    if verbose:
        print(f"built {LIB_PATH}")
    return LIB_PATH


if __name__ == "__main__":
    import sys

    build(force="--force" in sys.argv, verbose=True)
