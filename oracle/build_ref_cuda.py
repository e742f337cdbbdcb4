"""Build the reference's own CUDA extension for sm_100a into ``oracle/_ref/``.

Test infrastructure only.  It compiles the reference's four extension sources
(``csrc/bindings.cpp``, ``csrc/bgmv_shrink.cu``, ``csrc/bgmv_expand.cu``,
``csrc/gemv_fp16.cu``) where they lie, with the flags of the reference's
``setup.py`` (nvcc ``-O3 --use_fast_math``, g++ ``-O3``) plus the torch
extension defines, for ``compute_100a/sm_100a``, and links
``oracle/_ref/persona_ref_C.so``.  Nothing is copied.  The reference's own
build system is not run.

The library registers the reference's ``torch.ops.persona`` schemas, the
same namespace this package registers, so it is loaded only in a separate
process (``tests/ref_cuda_runner.py``).

    python oracle/build_ref_cuda.py [--reference DIR] [--force]
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
LIB = OUT_DIR / "persona_ref_C.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
SOURCES_CU = ["bgmv_shrink.cu", "bgmv_expand.cu", "gemv_fp16.cu"]
SOURCE_CPP = "bindings.cpp"


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"reference build step failed: {' '.join(cmd)}\n{r.stdout}")


def build(reference: Path, force: bool = False) -> Path:
    csrc = reference / "csrc"
    srcs = [csrc / s for s in SOURCES_CU] + [csrc / SOURCE_CPP]
    if not all(s.exists() for s in srcs):
        raise FileNotFoundError(f"reference sources not found under {csrc}")
    if LIB.exists() and not force and all(s.stat().st_mtime <= LIB.stat().st_mtime for s in srcs):
        return LIB
    import torch
    from torch.utils import cpp_extension as ce

    OUT_DIR.mkdir(parents=True, exist_ok=True)
    incs = ce.include_paths(device_type="cuda") if "device_type" in ce.include_paths.__code__.co_varnames \
        else ce.include_paths(cuda=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=persona_ref_C",
            "-DTORCH_API_INCLUDE_EXTENSION_H"]
    inc = []
    for i in incs + [sysconfig.get_paths()["include"]]:
        inc += ["-isystem", i]
    objs = []
    for s in SOURCES_CU:
        o = OUT_DIR / (Path(s).stem + ".o")
        # the defines torch's extension builder passes to nvcc, then the
        # reference's own nvcc flags
        _run([str(CUDA_HOME / "bin" / "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17",
              "-Xcompiler", "-fPIC", "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
              "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__", "--expt-relaxed-constexpr",
              "-O3", "--use_fast_math", *defs, *inc, "-c", str(csrc / s), "-o", str(o)])
        objs.append(o)
    o = OUT_DIR / "bindings.o"
    _run(["g++", "-O3", "-std=c++17", "-fPIC", *defs, *inc, "-c", str(csrc / SOURCE_CPP), "-o", str(o)])
    objs.append(o)
    torch_lib = Path(torch.__file__).parent / "lib"
    tmp = LIB.with_suffix(".tmp")
    _run(["g++", "-shared", "-o", str(tmp), *map(str, objs), "-L", str(torch_lib), "-lc10", "-lc10_cuda",
          "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-L", str(CUDA_HOME / "lib64"),
          "-lcudart"])
    os.replace(tmp, LIB)
    for ob in objs:
        ob.unlink()
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PERSONA_REFERENCE_DIR"),
                    required="PERSONA_REFERENCE_DIR" not in os.environ,
                    help="checkout of the reference repository (default: $PERSONA_REFERENCE_DIR)")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(Path(a.reference), a.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
