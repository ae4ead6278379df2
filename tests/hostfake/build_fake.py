"""Build the host-logic test double (test infrastructure only).

Compiles tests/hostfake/fake_fz.cpp into tests/hostfake/_build/libfusion_b200_hostfake.so and
links a copy of the pybind module (nova_b200/host/*.cpp) against it into the same
folder, so CPU tests can exercise the C++ host layer without a GPU.
"""
import pathlib
import subprocess
import sys
import sysconfig

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "_build"
EXT = OUT / ("fusion" + sysconfig.get_config_var("EXT_SUFFIX"))


def _stale(out, deps):
    return not out.exists() or any(d.stat().st_mtime > out.stat().st_mtime for d in deps)


def build() -> pathlib.Path:
    import pybind11

    OUT.mkdir(exist_ok=True)
    inc = ["-I" + str(ROOT / "include"), "-I" + str(ROOT / "nova_b200" / "host"),
           "-I" + pybind11.get_include(), "-I" + sysconfig.get_paths()["include"]]
    lib = OUT / "libfusion_b200_hostfake.so"
    src = HERE / "fake_fz.cpp"
    hdr = ROOT / "include" / "fusion_b200.h"
    if _stale(lib, [src, hdr]):
        subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", *inc,
                        str(src), "-o", str(lib)], check=True)
    host = sorted((ROOT / "nova_b200" / "host").glob("*.cpp"))
    deps = [lib, hdr, *host, *(ROOT / "nova_b200" / "host").glob("*.hpp")]
    if _stale(EXT, deps):
        subprocess.run(["g++", "-O1", "-std=c++20", "-fPIC", "-shared", "-fvisibility=hidden",
                        "-ffp-contract=off", *inc, *map(str, host), "-o", str(EXT),
                        "-L" + str(OUT), "-lfusion_b200_hostfake", "-Wl,-rpath,$ORIGIN"], check=True)
    return EXT


if __name__ == "__main__":
    print(build())
    sys.exit(0)
