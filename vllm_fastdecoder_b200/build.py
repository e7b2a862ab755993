"""Build the C-ABI library libfastdecode_b200.so for sm_100a with nvcc.

    python -m vllm_fastdecoder_b200.build          # incremental
    python -m vllm_fastdecoder_b200.build --force  # rebuild everything

Each csrc/*.cu is compiled to an object in _build/ (in parallel, rebuilt when
the source or any header is newer), then linked into _lib/ next to this file.
The library is plain CUDA C++ with an extern "C" surface (include/
fastdecode_b200.h); it links the shared CUDA runtime and nothing from torch.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIBDIR = PKG / "_lib"
LIBNAME = "libfastdecode_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin on PATH)")
    return cand


def _flags() -> list[str]:
    return ARCH + [
        "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        f"-I{INCLUDE}", f"-I{CSRC}",
    ]


def _newest_header() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, force: bool, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if not force and obj.exists():
        t = obj.stat().st_mtime
        if t >= src.stat().st_mtime and t >= _newest_header():
            return obj
    cmd = [nvcc()] + _flags() + ["-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    return obj


def library_path() -> Path:
    return LIBDIR / LIBNAME


def build_library(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    lib = library_path()
    if (not force and lib.exists()
            and lib.stat().st_mtime >= max(o.stat().st_mtime for o in objs)):
        return lib
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "shared", "-o", str(tmp)] + [str(o) for o in objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib)
    return lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas register/spill report")
    a = ap.parse_args()
    print(build_library(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
