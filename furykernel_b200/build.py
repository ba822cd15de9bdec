"""Builds libfurykernel_cuda.so in-tree for sm_100a with nvcc.

Strict arithmetic: --fmad=false (no contraction but explicit fma, the
reference's `Strict` math, src/FuryKernel/Backend.hs:179-200), IEEE division
and square root, no fast math.
"""

from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libfurykernel_cuda.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs() -> tuple[str, str]:
    """NCCL's headers and library: the copy torch loads, so that one NCCL
    serves the process."""
    try:
        import nvidia.nccl  # type: ignore

        base = list(nvidia.nccl.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except ImportError:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    deps.append(os.path.join(HERE, "..", "include", "furykernel_cuda.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _compile(src: str, obj: str, inc: str, ptxas_v: bool, verbose: bool) -> None:
    """One translation unit, written under a temporary name and then renamed,
    so that an interrupted compile leaves no object that looks current."""
    tmp = f"{obj[:-2]}.{os.getpid()}.tmp.o"
    cmd = ["nvcc", *ARCH, "-O3", "-lineinfo", "--fmad=false", "-std=c++17", "-Xcompiler", "-fPIC",
           "-I", inc, "-c", src, "-o", tmp]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, obj)


def build(verbose: bool = False, ptxas_v: bool = False) -> str:
    from concurrent.futures import ThreadPoolExecutor

    os.makedirs(OUT_DIR, exist_ok=True)
    inc, lib = nccl_dirs()
    deps = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        [os.path.join(HERE, "..", "include", "furykernel_cuda.h")]
    newest_dep = max(os.path.getmtime(p) for p in deps)
    objs, stale_srcs = [], []
    for src in sources():
        obj = os.path.join(OUT_DIR, os.path.basename(src)[:-3] + ".o")
        if not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), newest_dep):
            stale_srcs.append((src, obj))
        objs.append(obj)
    # nvcc's front end and ptxas each run on one core: the stale units
    # compile side by side, the build taking about as long as the longest.
    if stale_srcs:
        with ThreadPoolExecutor(max_workers=max(1, min(len(stale_srcs), os.cpu_count() or 1))) as pool:
            for f in [pool.submit(_compile, s, o, inc, ptxas_v, verbose) for s, o in stale_srcs]:
                f.result()
    cmd = ["nvcc", *ARCH, "-shared", "-o", LIB, *objs, "-L", lib, "-l:libnccl.so.2", "-Xlinker", f"-rpath,{lib}"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    return LIB


HOST = os.path.join(HERE, "host")
HOST_LIB = os.path.join(OUT_DIR, "libfurykernel_host.so")


def build_host(verbose: bool = False) -> str:
    """libfurykernel_host.so: the programs, the planner and the lowering in
    C++ (g++, no CUDA), behind include/furykernel_host.h."""
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(HOST, "*.cc")))
    deps = srcs + glob.glob(os.path.join(HOST, "*.h")) + [os.path.join(HERE, "..", "include", "furykernel_host.h")]
    if os.path.exists(HOST_LIB) and all(os.path.getmtime(d) <= os.path.getmtime(HOST_LIB) for d in deps):
        return HOST_LIB
    # Several processes (the ranks of a tensor-parallel run) may find the
    # library stale at once: each builds its own file and renames it into
    # place, so that no process loads a half-written library.
    tmp = f"{HOST_LIB}.{os.getpid()}.tmp"
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", "-Wno-unused-parameter",
           "-fvisibility=hidden", *srcs, "-o", tmp]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    try:
        subprocess.run(cmd, check=True)
        os.replace(tmp, HOST_LIB)
    finally:
        if os.path.exists(tmp):
            os.remove(tmp)
    return HOST_LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_v="-v" in sys.argv))
    print(build_host(verbose=True))
