"""Build the native libraries in-tree.

1. ``fused_hoad/libfused_hoad_b200.so`` -- the CUDA kernels and the C ABI of
   ``include/fused_hoad_b200.h``, compiled by nvcc for sm_100a only
   (``-gencode arch=compute_100a,code=sm_100a``), linked against the shared CUDA runtime.
2. ``fused_hoad/_C*.so`` -- the torch.utils.cpp_extension binding (``csrc/bindings.cpp``),
   linked against (1) with an ``$ORIGIN`` rpath so both travel together.

Usage: ``python expanded-gpu-optimization_b200/build.py [--force]``. nvcc cross-compiles, so
this runs without a GPU. ``-Xptxas -v`` output (registers, spills, shared memory) goes to
``_build/ptxas.txt``.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
PKG = HERE / "fused_hoad"
BUILD = HERE / "_build"
INCLUDE = HERE.parent / "include"
LIB = PKG / "libfused_hoad_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O3",
    "-Xptxas",
    "-v",
    f"-I{INCLUDE}",
]
CU_SOURCES = [
    "forward_fp32.cu", "forward_tc.cu", "backward_fp32.cu", "backward_tc.cu", "adam.cu",
    "collective.cu", "capi.cu", "noalloc.cu", "biharmonic.cu",
]


def _headers() -> list[Path]:
    return [*CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    newest = max(s.stat().st_mtime for s in sources)
    return target.stat().st_mtime < newest


def _compile(src: Path, force: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    if force or _stale(obj, [src, *_headers()]):
        proc = subprocess.run(
            [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)],
            capture_output=True,
            text=True,
        )
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stdout}\n{proc.stderr}")
        return obj, proc.stderr
    return obj, ""


def build_native(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = [CSRC / name for name in CU_SOURCES]
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(sources)) as pool:
        results = list(pool.map(lambda s: _compile(s, force), sources))
    logs = [log for _, log in results if log]
    if logs:
        (BUILD / "ptxas.txt").write_text("\n".join(logs))
    objects = [obj for obj, _ in results]
    if force or _stale(LIB, objects):
        subprocess.check_call(
            [NVCC, *ARCH, "-shared", "-cudart", "shared", "-o", str(LIB), *map(str, objects)]
        )
    return LIB


def build_binding(force: bool = False) -> Path:
    existing = sorted(PKG.glob("_C*.so"))
    sources = [CSRC / "bindings.cpp", LIB, *INCLUDE.glob("*.h")]
    if existing and not force and not _stale(existing[0], sources):
        return existing[0]
    proc = subprocess.run(
        [sys.executable, str(Path(__file__).resolve()), "--setup-binding"],
        cwd=str(HERE),
        capture_output=True,
        text=True,
    )
    if proc.returncode != 0:
        raise RuntimeError(f"binding build failed:\n{proc.stdout[-4000:]}\n{proc.stderr[-4000:]}")
    built = sorted(PKG.glob("_C*.so"))
    if not built:
        raise RuntimeError("binding build produced no library")
    return built[0]


def _setup_binding() -> None:
    from setuptools import setup
    from torch.utils.cpp_extension import BuildExtension, CUDAExtension

    setup(
        name="fused_hoad_b200_binding",
        ext_modules=[
            CUDAExtension(
                name="fused_hoad._C",
                sources=["csrc/bindings.cpp"],
                include_dirs=[str(INCLUDE)],
                library_dirs=[str(PKG)],
                libraries=["fused_hoad_b200"],
                extra_compile_args={"cxx": ["-O3"]},
                extra_link_args=["-Wl,-rpath,$ORIGIN"],
            )
        ],
        cmdclass={"build_ext": BuildExtension},
        package_dir={"": "."},
        script_args=["build_ext", "--inplace", "--build-temp", str(BUILD / "binding")],
    )


def build(force: bool = False) -> list[Path]:
    return [build_native(force), build_binding(force)]


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--setup-binding", action="store_true", help=argparse.SUPPRESS)
    args = parser.parse_args()
    if args.setup_binding:
        _setup_binding()
        return
    for path in build(args.force):
        print(path)


if __name__ == "__main__":
    main()
