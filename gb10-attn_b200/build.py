"""Build recipe for the B200 paged-attention library (in-tree, sm_100a only).

Produces, next to the Python package (so the files travel with the tree):

* ``pa_b200/libpa_b200.so`` -- the C-ABI library (``include/pa_b200.h``):
  hand-written CUDA for ``-gencode arch=compute_100a,code=sm_100a``, no torch.
* ``pa_b200/_pa_b200_torch.so`` -- the torch shim (``csrc/torch_shim.cpp``)
  exporting the reference's C++ operator signatures, linked against the
  C-ABI library.

Object files go to ``_build/`` and are rebuilt only when a source or header
is newer.  nvcc cross-compiles, so this runs without a GPU.

Usage: ``python gb10-attn_b200/build.py [--force] [--jobs N]``
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent            # gb10-attn_b200/
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
OUT_DIR = PKG_ROOT / "pa_b200"
BUILD = PKG_ROOT / "_build"
INCLUDE = REPO / "include"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
                     f"-I{INCLUDE}"]

CU_SOURCES = ["abi.cu", "decode.cu", "decode_f16.cu", "decode_bf16.cu", "decode_f32.cu",
              "decode_f64.cu", "decode_e4m3.cu", "decode_static.cu", "write_kv.cu",
              "prefill.cu", "prefill_tc.cu", "prefill_pair.cu", "peer_merge.cu"]
LIB = OUT_DIR / "libpa_b200.so"
SHIM = OUT_DIR / "_pa_b200_torch.so"


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths if p.exists()), default=0.0)


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")


def _compile_cu(src: Path, force: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, _newest(_headers())):
        _run([NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    return obj


def build_lib(force: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = [CSRC / s for s in CU_SOURCES if (CSRC / s).exists()]
    with ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile_cu(s, force), srcs))
    if force or not LIB.exists() or LIB.stat().st_mtime < _newest(objs):
        tmp = LIB.with_suffix(f".so.{os.getpid()}.tmp")
        _run([NVCC, *ARCH, "-shared", "-cudart", "shared", "-o", str(tmp), *map(str, objs),
              "-Xlinker", f"-rpath,{CUDA_HOME / 'lib64'}", "-Xlinker", "-soname,libpa_b200.so"])
        os.replace(tmp, LIB)
    return LIB


def build_shim(force: bool = False) -> Path:
    import torch.utils.cpp_extension as ce

    src = CSRC / "torch_shim.cpp"
    obj = BUILD / "torch_shim.o"
    deps = [src, *_headers()]
    if force or not obj.exists() or obj.stat().st_mtime < _newest(deps):
        inc = [f"-I{p}" for p in ce.include_paths("cuda")] + [
            f"-I{sysconfig.get_paths()['include']}", f"-I{INCLUDE}"]
        abi = int(__import__("torch")._C._GLIBCXX_USE_CXX11_ABI)
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", *inc,
              f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_pa_b200_torch",
              "-DTORCH_API_INCLUDE_EXTENSION_H", "-c", str(src), "-o", str(obj)])
    if force or not SHIM.exists() or SHIM.stat().st_mtime < max(obj.stat().st_mtime, LIB.stat().st_mtime):
        libdirs = ce.library_paths("cuda")
        tmp = SHIM.with_suffix(f".so.{os.getpid()}.tmp")
        _run(["g++", "-shared", "-o", str(tmp), str(obj), f"-L{OUT_DIR}", "-lpa_b200",
              *[f"-L{d}" for d in libdirs], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
              "-ltorch_cuda", "-ltorch_python", "-lcudart",
              "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{d}" for d in libdirs]])
        os.replace(tmp, SHIM)
    return SHIM


def build(force: bool = False, jobs: int | None = None) -> None:
    build_lib(force, jobs)
    build_shim(force)


def clean() -> None:
    shutil.rmtree(BUILD, ignore_errors=True)
    for p in (LIB, SHIM):
        p.unlink(missing_ok=True)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--clean", action="store_true")
    a = ap.parse_args()
    if a.clean:
        clean()
    build(a.force, a.jobs)
    print(LIB)
    print(SHIM)
