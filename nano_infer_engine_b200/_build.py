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
    "nie_linear.cu",
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


EXT_SOURCE = CSRC / "nie_torch_ext.cpp"
EXT_NAME = "_nie_torch_ext"
EXT_PATH = PKG_DIR / (EXT_NAME + ".so")


def build_ext(force: bool = False, verbose: bool = False) -> Path:
    """Compile the torch C++ extension (the per-layer loop of a ragged step) with g++.

    It links against ``libnie_b200.so`` beside it (rpath ``$ORIGIN``) and
    against the installed torch, so it must be rebuilt with torch.
    """
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    inputs = [EXT_SOURCE, LIB_PATH, *INCLUDE_DIR.glob("*.h"), Path(torch.__file__)]
    if not force and EXT_PATH.exists() and all(p.stat().st_mtime <= EXT_PATH.stat().st_mtime for p in inputs):
        return EXT_PATH
    includes = [*cpp_extension.include_paths(device_type="cuda"), sysconfig.get_paths()["include"], str(INCLUDE_DIR)]
    lib_dirs = [str(PKG_DIR), *cpp_extension.library_paths(device_type="cuda")]
    torch_lib = str(Path(torch.__file__).resolve().parent / "lib")
    tmp = EXT_PATH.with_suffix(".so.tmp")
    cmd = [
        os.environ.get("CXX", "g++"),
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
        f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        *(f"-I{d}" for d in includes),
        str(EXT_SOURCE),
        "-o",
        str(tmp),
        *(f"-L{d}" for d in lib_dirs),
        "-lnie_b200",
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_cuda",
        "-ltorch_python",
        "-Wl,-rpath,$ORIGIN",
        f"-Wl,-rpath,{torch_lib}",
    ]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"g++ failed for {EXT_SOURCE.name}:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, EXT_PATH)
    if verbose:
        print(f"built {EXT_PATH}")
    return EXT_PATH


if __name__ == "__main__":
    import sys

    build(force="--force" in sys.argv, verbose=True)
    build_ext(force="--force" in sys.argv, verbose=True)
