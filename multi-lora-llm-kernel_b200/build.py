"""Build the in-tree native libraries of the persona package.

* ``persona/libpersona_bgmv.so``: the CUDA kernels and their ``extern "C"``
  API (``include/persona_bgmv.h``), compiled by nvcc for sm_100a only,
  static CUDA runtime, no torch dependency.
* ``persona/_C<ext>``: the torch op registrations (``csrc/bindings.cpp``)
  over that C API, compiled by g++ against the installed torch.

    python multi-lora-llm-kernel_b200/build.py [--force] [--verbose]

Outputs are rebuilt only when a source or header is newer than them.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO / "include"
OUT = PKG_ROOT / "persona"
BUILD = REPO / "_build" / "persona"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_SOURCES = ["capi.cu", "bgmv_plan.cu", "bgmv_split.cu", "sgmv_tcgen05.cu", "simple_kernels.cu",
              "noalloc.cu", "nf4.cu", "decode_ops.cu", "bgmv_small.cu"]
LIB = OUT / "libpersona_bgmv.so"
EXT = OUT / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def _deps() -> list[Path]:
    return sorted(list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)])


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}")
    if verbose and r.stdout.strip():
        print(r.stdout, flush=True)


def build_lib(verbose: bool = False, force: bool = False) -> Path:
    deps = _deps()
    if not force and not _stale(LIB, deps):
        return LIB
    BUILD.mkdir(parents=True, exist_ok=True)
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                    "-I", str(INCLUDE), "-I", str(CSRC)]
    objs = []
    jobs = []
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(CU_SOURCES), os.cpu_count() or 1))) as ex:
        for src in CU_SOURCES:
            obj = BUILD / (Path(src).stem + ".o")
            objs.append(obj)
            cmd = [NVCC, *flags, "-c", str(CSRC / src), "-o", str(obj)]
            jobs.append(ex.submit(_run, cmd, verbose))
        for j in jobs:
            j.result()
    tmp = LIB.with_suffix(".so.tmp")
    _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-Xlinker", "--no-undefined",
          "-lcudart_static", "-ldl", "-lrt", "-lpthread"], verbose)
    os.replace(tmp, LIB)
    return LIB


def build_ext(verbose: bool = False, force: bool = False) -> Path:
    deps = _deps() + [LIB]
    if not force and not _stale(EXT, deps):
        return EXT
    import torch
    from torch.utils import cpp_extension as ce

    incs = ce.include_paths(device_type="cuda") if "device_type" in ce.include_paths.__code__.co_varnames \
        else ce.include_paths(cuda=True)
    torch_lib = Path(torch.__file__).parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-shared", str(CSRC / "bindings.cpp"),
           "-o", str(EXT.with_suffix(".tmp")),
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-I", str(INCLUDE),
           "-I", sysconfig.get_paths()["include"]]
    for i in incs:
        cmd += ["-isystem", i]
    cmd += ["-L", str(torch_lib), "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            "-ltorch_python", "-L", str(OUT), "-lpersona_bgmv",
            "-L", str(CUDA_HOME / "lib64"), "-lcudart", "-Wl,-rpath,$ORIGIN"]
    _run(cmd, verbose)
    os.replace(EXT.with_suffix(".tmp"), EXT)
    return EXT


def build(verbose: bool = False, force: bool = False) -> None:
    if shutil.which(NVCC) is None and not Path(NVCC).exists():
        raise RuntimeError(f"nvcc not found at {NVCC}")
    build_lib(verbose, force)
    build_ext(verbose, force)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    build(a.verbose, a.force)
    print(f"built {LIB.name} and {EXT.name}")


if __name__ == "__main__":
    sys.exit(main())
