"""Compile the reference's own code, from its sources, into oracle/_ref/.

TEST INFRASTRUCTURE ONLY (the checker, never the product).  Nothing is copied:
the compilers read the files where they lie under the reference checkout
($GB10_REF, else a checkout named ``reference`` beside this repository).
Outputs go to oracle/_ref/ only (git-ignored; it travels to the GPU box with
the tree).

* libref_arm_scalar.so -- gb10-attn arm_cpu/src/scalar.cpp (the reference's
  scalar dot / scores / softmax lane) + ref_arm_shim.cpp, with the reference's
  flags for that file (-O3 -fno-tree-vectorize, arm_cpu/CMakeLists.txt:21-25).
* gb10_ref_kernels.so -- gb10-attn kernels/paged_attn_{v1,v2,v3,prefill,wmma}.cu
  unchanged, with the reference's flags (-O3 --use_fast_math,
  kernels/paged_attn_v3.h:5-7) for -gencode arch=compute_100a,code=sm_100a,
  + ref_kernels_bind.cpp.  Runs only on a GPU; used by -m gpu tests and by
  tests/golden/make_golden.py.
* arm_attn_bench -- the reference's own CPU microbenchmark
  (arm_cpu/src/{bench,scalar,neon,sve,features}.cpp, flags of
  arm_cpu/CMakeLists.txt: -O3, -fno-tree-vectorize on scalar.cpp).  bench.py's
  CPU-baseline leg runs ``--backend scalar --tokens 2048 --dim 64`` (scores +
  softmax of one head, no V, no paging) beside the scalar decode restatement.

The reference's only full CPU paged decode (cpu_reference in
rocm/hip/paged_attn_v1_hip.cpp) sits in a HIP translation unit that needs the
ROCm headers, so it is not buildable here; pa_oracle.c restates it.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
REF = Path(os.environ.get("GB10_REF", str(HERE.parent.parent / "reference")))
KERNELS = ["paged_attn_v1", "paged_attn_v2", "paged_attn_v3", "paged_attn_prefill",
           "paged_attn_wmma"]


def available() -> bool:
    return (REF / "kernels" / "paged_attn_v3.cu").is_file()


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(" ".join(map(str, cmd)) + "\n" + r.stdout + r.stderr)
        raise RuntimeError("reference build failed")


def build_arm_scalar(force: bool = False) -> Path:
    out = OUT / "libref_arm_scalar.so"
    src = REF / "arm_cpu" / "src" / "scalar.cpp"
    if out.exists() and not force:
        return out
    OUT.mkdir(exist_ok=True)
    _run(["g++", "-O3", "-std=c++20", "-fno-tree-vectorize", "-fPIC", "-shared",
          f"-I{REF / 'arm_cpu' / 'include'}", str(src), str(HERE / "ref_arm_shim.cpp"),
          "-o", str(out)])
    return out


def build_arm_bench(force: bool = False) -> Path:
    out = OUT / "arm_attn_bench"
    if out.exists() and not force:
        return out
    OUT.mkdir(exist_ok=True)
    obj_dir = OUT / "obj_arm"
    obj_dir.mkdir(exist_ok=True)
    src = REF / "arm_cpu" / "src"
    objs = []
    for name in ("bench", "scalar", "neon", "sve", "features"):
        o = obj_dir / f"{name}.o"
        extra = ["-fno-tree-vectorize"] if name == "scalar" else []
        _run(["g++", "-O3", "-std=c++20", *extra, f"-I{REF / 'arm_cpu' / 'include'}",
              "-c", str(src / f"{name}.cpp"), "-o", str(o)])
        objs.append(o)
    _run(["g++", "-o", str(out), *map(str, objs)])
    for o in objs:
        o.unlink(missing_ok=True)
    return out


def build_cuda_kernels(force: bool = False) -> Path:
    import torch.utils.cpp_extension as ce
    out = OUT / "gb10_ref_kernels.so"
    if out.exists() and not force:
        return out
    OUT.mkdir(exist_ok=True)
    obj_dir = OUT / "obj"
    obj_dir.mkdir(exist_ok=True)
    inc = [f"-I{p}" for p in ce.include_paths("cuda")] + [f"-I{sysconfig.get_paths()['include']}"]
    abi = int(__import__("torch")._C._GLIBCXX_USE_CXX11_ABI)
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
            "-DTORCH_EXTENSION_NAME=gb10_ref_kernels"]
    nvcc = str(Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc")

    def cu(name):
        o = obj_dir / f"{name}.o"
        _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--use_fast_math",
              "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
              "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__",
              *inc, *defs, "-c", str(REF / "kernels" / f"{name}.cu"), "-o", str(o)])
        return o

    def bind():
        o = obj_dir / "bind.o"
        _run(["g++", "-O2", "-std=c++17", "-fPIC", *inc, *defs, f"-I{REF / 'kernels'}",
              "-c", str(HERE / "ref_kernels_bind.cpp"), "-o", str(o)])
        return o

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        futs = [ex.submit(cu, k) for k in KERNELS] + [ex.submit(bind)]
        objs = [f.result() for f in futs]
    libdirs = ce.library_paths("cuda")
    _run(["g++", "-shared", "-o", str(out), *map(str, objs), *[f"-L{d}" for d in libdirs],
          "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
          "-lcudart", *[f"-Wl,-rpath,{d}" for d in libdirs]])
    for o in objs:
        o.unlink(missing_ok=True)
    return out


def build(force: bool = False) -> bool:
    """Build both when the reference sources are present; False otherwise."""
    if not available():
        return False
    build_arm_scalar(force)
    build_arm_bench(force)
    build_cuda_kernels(force)
    return True


if __name__ == "__main__":
    print("built" if build("--force" in sys.argv) else "reference sources not found")
