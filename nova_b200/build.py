"""Build the in-tree native libraries of nova_b200.

* ``nova_b200/libfusion_b200.so`` -- the CUDA kernels and the C ABI declared in
  ``include/fusion_b200.h``, compiled for sm_100a only.
* ``nova_b200/fusion<ext>`` -- the pybind11 module ``fusion`` (Fusion's Python
  API: Tensor, factory, Random, grad_tape, autodiff), C++ host code over the C ABI.

Run ``python -m nova_b200.build`` (or ``__graft_entry__.build()``). Objects are
rebuilt only when a source or header is newer than the output.
"""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = PKG / "host"
INCLUDE = ROOT / "include"
OBJ = PKG / "_build"
CUDA_HOME = pathlib.Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB = PKG / "libfusion_b200.so"
EXT = PKG / ("fusion" + sysconfig.get_config_var("EXT_SUFFIX"))

NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--fmad=false",
    "-I" + str(INCLUDE), "-I" + str(CSRC), "-Xptxas", "-warn-spills",
]


def _nccl_dirs():
    """NCCL header and library used by the collective entry points.

    Prefer the NCCL wheel in the Python environment: it is the copy torch loads, and
    two NCCL builds cannot coexist in one process (they share the soname
    libnccl.so.2), so linking the same one keeps `import torch` working in either
    import order."""
    site = pathlib.Path(sysconfig.get_paths()["purelib"]) / "nvidia" / "nccl"
    if (site / "include" / "nccl.h").exists() and (site / "lib" / "libnccl.so.2").exists():
        return site / "include", site / "lib"
    return pathlib.Path("/usr/include"), pathlib.Path("/usr/lib/x86_64-linux-gnu")


def _stale(out: pathlib.Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(pathlib.Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd[:3]) + " ...")
    if verbose and (r.stderr.strip()):
        sys.stderr.write(r.stderr)


def _embed_kernel_source() -> pathlib.Path:
    """Write the GEMM kernels' device source as a C++ string literal, the text the
    library hands NVRTC when it compiles a GEMM with a fused epilogue (rewritten only
    when the header changed)."""
    src = (CSRC / "fz_gemm_kernels.cuh").read_text()
    delim = "FZSRC"
    assert ")" + delim + '"' not in src
    out = OBJ / "fz_gemm_kernels.inc"
    text = 'R"' + delim + "(" + src + ")" + delim + '"\n'
    if not out.exists() or out.read_text() != text:
        out.write_text(text)
    return out


def build_lib(verbose: bool = False, jobs: int = 8) -> pathlib.Path:
    OBJ.mkdir(exist_ok=True)
    inc = _embed_kernel_source()
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + [INCLUDE / "fusion_b200.h", inc]
    srcs = sorted(CSRC.glob("*.cu"))
    nccl_inc, nccl_lib = _nccl_dirs()
    jobs_list = []
    objs = []
    for src in srcs:
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers]):
            jobs_list.append([NVCC, *NVCC_FLAGS, "-I" + str(OBJ), "-I" + str(nccl_inc), "-c", str(src),
                              "-o", str(obj)])
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(lambda c: _run(c, verbose), jobs_list))
    if jobs_list or _stale(LIB, objs):
        nccl_so = nccl_lib / "libnccl.so"
        nccl_link = ["-L" + str(nccl_lib), "-lnccl"] if nccl_so.exists() else [
            "-L" + str(nccl_lib), "-Xlinker", "-l:libnccl.so.2"]
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), *nccl_link, "-lnvrtc",
              "-Xlinker", "-rpath," + str(nccl_lib) + ":" + str(CUDA_HOME / "lib64")], verbose)
    return LIB


def build_ext(verbose: bool = False, jobs: int = 8) -> pathlib.Path | None:
    srcs = sorted(HOST.glob("*.cpp"))
    if not srcs:
        return None
    import pybind11

    OBJ.mkdir(exist_ok=True)
    headers = list(HOST.glob("*.hpp")) + [INCLUDE / "fusion_b200.h"]
    pyinc = sysconfig.get_paths()["include"]
    flags = ["-O2", "-std=c++20", "-fPIC", "-fvisibility=hidden", "-ffp-contract=off",
             "-I" + str(INCLUDE), "-I" + str(HOST), "-I" + pybind11.get_include(), "-I" + pyinc,
             "-I" + str(CUDA_HOME / "include")]
    jobs_list, objs = [], []
    for src in srcs:
        obj = OBJ / ("host_" + src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers]):
            jobs_list.append(["g++", *flags, "-c", str(src), "-o", str(obj)])
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(lambda c: _run(c, verbose), jobs_list))
    if jobs_list or _stale(EXT, [*objs, LIB]):
        _run(["g++", "-shared", "-o", str(EXT), *map(str, objs), "-L" + str(PKG), "-lfusion_b200",
              "-Wl,-rpath,$ORIGIN"], verbose)
    return EXT


def build(verbose: bool = False) -> None:
    if not shutil.which(NVCC) and not pathlib.Path(NVCC).exists():
        raise RuntimeError("nvcc not found at " + NVCC)
    build_lib(verbose)
    build_ext(verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
