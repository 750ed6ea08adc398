"""In-tree native build of the framework (no pip install, no JIT cache).

Three artefacts are produced with one ninja file:

* ``opengda_b200/lib/libgicc.so`` -- the native runtime: socket bootstrap, symmetric
  memory (CUDA VMM + NVLS multicast), Runtime/Barrier/AM host classes and every
  sm_100a kernel (``csrc/src/*.cpp``, ``csrc/kernels/*.cu``).  It has no torch
  dependency, so C++ programs link it directly (the reference ships ``libgicc.so``
  the same way, src/CMakeLists.txt:37-39).
* ``opengda_b200/_C*.so`` -- the thin pybind/torch binding (``csrc/bindings``).
* ``opengda_b200/bin/*`` -- native benchmark/app executables (``csrc/apps``), the
  counterparts of the reference's ``examples/gicc/*.cu`` programs.

Every CUDA translation unit is compiled for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = ROOT / "csrc"
BUILD = ROOT / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _torch_flags():
    import torch
    from torch.utils import cpp_extension as ce

    inc = ce.include_paths(device_type="cuda")
    libs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = [f"-I{p}" for p in inc] + [
        f"-I{sysconfig.get_paths()['include']}",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_EXTENSION_NAME=_C",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
    ]
    ldflags = [f"-L{p}" for p in libs] + [f"-Wl,-rpath,{libs[0]}"] + [
        "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
    ]
    return cflags, ldflags


def _ninja_file(debug_checks: bool) -> str:
    nvcc = str(CUDA_HOME / "bin" / "nvcc")
    inc = f"-I{CSRC / 'include'} -I{CUDA_HOME / 'include'}"
    checks = " -DGICC_CHECKS=1" if debug_checks else ""
    nvflags = (
        f"-std=c++17 -O3 {' '.join(ARCH)} -lineinfo -Xcompiler -fPIC,-fvisibility=hidden "
        f"--expt-relaxed-constexpr -diag-suppress=177 -Xptxas -v {inc}{checks}"
    )
    cxxflags = f"-std=c++17 -O2 -fPIC -fvisibility=hidden -Wall -Wno-unused-function {inc}{checks}"
    tcflags, tldflags = _torch_flags()
    ext_suffix = sysconfig.get_config_var("EXT_SUFFIX")

    srcs_cpp = sorted((CSRC / "src").glob("*.cpp"))
    srcs_cu = sorted((CSRC / "kernels").glob("*.cu"))
    binds = sorted((CSRC / "bindings").glob("*.cpp"))
    apps = sorted((CSRC / "apps").glob("*.cu"))

    lines = [
        "ninja_required_version = 1.3",
        f"nvcc = {nvcc}",
        "cxx = g++",
        f"nvflags = {nvflags}",
        f"cxxflags = {cxxflags}",
        f"tflags = -std=c++17 -O2 -fPIC -I{CSRC / 'include'} -I{CUDA_HOME / 'include'} {' '.join(tcflags)}",
        "rule nvcc",
        "  command = $nvcc $nvflags -MD -MF $out.d -c $in -o $out > $out.ptxas.log 2>&1 || (cat $out.ptxas.log; exit 1)",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = NVCC $in",
        "rule cxx",
        "  command = $cxx $cxxflags -MD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CXX $in",
        "rule tcxx",
        "  command = $cxx $tflags -MD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CXX(torch) $in",
        "rule solink",
        "  command = $nvcc -shared $in -o $out $ldflags",
        "  description = LINK $out",
        "rule tlink",
        "  command = $cxx -shared $in -o $out $ldflags",
        "  description = LINK $out",
        "rule applink",
        "  command = $nvcc $in -o $out $ldflags",
        "  description = LINK $out",
    ]
    objs = []
    for s in srcs_cpp:
        o = BUILD / "obj" / (s.stem + ".o")
        lines.append(f"build {o}: cxx {s}")
        objs.append(o)
    for s in srcs_cu:
        o = BUILD / "obj" / (s.stem + ".cu.o")
        lines.append(f"build {o}: nvcc {s}")
        objs.append(o)
    lib = PKG / "lib" / "libgicc.so"
    lines.append(f"build {lib}: solink {' '.join(map(str, objs))}")
    lines.append(f"  ldflags = {ARCH[0]} {ARCH[1]} -cudart static -lpthread -Xlinker -soname=libgicc.so")

    bobjs = []
    for s in binds:
        o = BUILD / "obj" / ("bind_" + s.stem + ".o")
        lines.append(f"build {o}: tcxx {s}")
        bobjs.append(o)
    ext = PKG / f"_C{ext_suffix}"
    lines.append(f"build {ext}: tlink {' '.join(map(str, bobjs))} | {lib}")
    lines.append(
        f"  ldflags = -L{PKG / 'lib'} -lgicc -Wl,-rpath,'$$ORIGIN/lib' {' '.join(tldflags)} "
    )
    for s in apps:
        exe = PKG / "bin" / s.stem
        lines.append(f"build {exe}: applink {s} | {lib}")
        lines.append(
            f"  ldflags = {nvflags} -L{PKG / 'lib'} -lgicc -Xlinker -rpath,'$$ORIGIN/../lib'"
        )
    return "\n".join(lines) + "\n"


def build(verbose: bool = False, debug_checks: bool = False) -> None:
    """Compile every native artefact in place (sm_100a).  Raises on failure."""
    if shutil.which("ninja") is None:
        import ninja  # noqa: F401  (pip ninja puts the binary on PATH via its module)
    BUILD.mkdir(exist_ok=True)
    (BUILD / "obj").mkdir(exist_ok=True)
    (PKG / "lib").mkdir(exist_ok=True)
    (PKG / "bin").mkdir(exist_ok=True)
    nf = BUILD / "build.ninja"
    text = _ninja_file(debug_checks)
    if not nf.exists() or nf.read_text() != text:
        nf.write_text(text)
    jobs = str(max(2, os.cpu_count() or 2))
    cmd = [shutil.which("ninja") or "ninja", "-C", str(BUILD), "-j", jobs]
    if verbose:
        cmd.append("-v")
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        out = (res.stdout or "") + (res.stderr or "")
        raise RuntimeError("native build failed:\n" + out[-8000:])


def ptxas_report() -> str:
    """Concatenated ``-Xptxas -v`` output (registers, spills, smem) of every kernel TU."""
    logs = sorted((BUILD / "obj").glob("*.ptxas.log"))
    return "\n".join(f"== {p.name}\n{p.read_text()}" for p in logs)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print("built", PKG / "lib" / "libgicc.so")
