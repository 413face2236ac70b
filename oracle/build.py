"""Build the checkers (TEST INFRASTRUCTURE ONLY).

* ``oracle/_build/libjet64.so``: the FP64 C restatement in ``oracle/c/jet64.c`` (gcc).
* ``oracle/_ref/fused_hoad_ref_C*.so``: the reference's own CUDA extension, compiled for
  sm_100a directly from its three source files where they lie in the read-only reference
  checkout (``csrc/bindings.cpp``, ``csrc/fused_residual.cu``, ``csrc/fused_backward.cu``).
  The reference's setup.py is not run; this recipe compiles the same files with
  ``torch.utils.cpp_extension`` under a module name of its own so it can sit beside the
  shipped ``fused_hoad._C``. Only built when the reference checkout is present (in the
  build container); the GPU box uses the prebuilt file that travels with the tree.

Usage: ``python -m oracle.build [--no-ref]``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
BUILD = ORACLE / "_build"
REF_OUT = ORACLE / "_ref"
# The reference checkout: FUSED_HOAD_REFERENCE, else a "reference" directory beside this
# repository. Absent (as on a GPU box), the prebuilt oracle/_ref library is used as is.
REFERENCE_ROOT = Path(
    os.environ.get("FUSED_HOAD_REFERENCE", str(ORACLE.parent.parent / "reference"))
)
REF_MODULE = "fused_hoad_ref_C"


def build_c_oracle(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    src = ORACLE / "c" / "jet64.c"
    out = BUILD / "libjet64.so"
    if force or not out.exists() or out.stat().st_mtime < src.stat().st_mtime:
        subprocess.check_call(
            ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-o", str(out), str(src), "-lm"]
        )
    return out


def reference_sources() -> list[Path]:
    csrc = REFERENCE_ROOT / "csrc"
    return [csrc / "bindings.cpp", csrc / "fused_residual.cu", csrc / "fused_backward.cu"]


def ref_library() -> Path | None:
    found = sorted(REF_OUT.glob(f"{REF_MODULE}*.so"))
    return found[0] if found else None


def build_reference(force: bool = False) -> Path | None:
    sources = reference_sources()
    if not all(s.exists() for s in sources):
        return ref_library()
    existing = ref_library()
    newest = max(s.stat().st_mtime for s in sources)
    if existing is not None and not force and existing.stat().st_mtime >= newest:
        return existing
    from torch.utils import cpp_extension

    work = REF_OUT / "build"
    work.mkdir(parents=True, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    cpp_extension.load(
        name=REF_MODULE,
        sources=[str(s) for s in sources],
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", "-lineinfo"],
        build_directory=str(work),
        verbose=False,
    )
    built = sorted(work.glob(f"{REF_MODULE}*.so"))
    if not built:
        raise RuntimeError("reference extension build produced no library")
    target = REF_OUT / built[0].name
    shutil.copy2(built[0], target)
    shutil.rmtree(work, ignore_errors=True)
    return target


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--no-ref", action="store_true", help="skip the reference CUDA build")
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build_c_oracle(args.force))
    if not args.no_ref:
        print(build_reference(args.force))


if __name__ == "__main__":
    sys.exit(main())
