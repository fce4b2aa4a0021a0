"""Build libk3moe.so (every sm_100a kernel + the C ABI) in-tree with nvcc."""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc", "capi.cu")
OUT = os.path.join(HERE, "libk3moe.so")
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-shared",
              "-Xcompiler", "-fPIC", "-Xptxas", "-v"]


def sources():
    d = os.path.join(HERE, "csrc")
    return [os.path.join(d, f) for f in sorted(os.listdir(d))] + [os.path.join(HERE, "..", "include", "k3moe.h")]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(s) <= t for s in sources())


CUBIN = os.path.join(HERE, "k3moe_module.cubin")


def build_cubin(nvcc: str) -> str:
    """The drop-in kernel module (csrc/module.cu: the extern "C" entries with the reference's names)."""
    cmd = [nvcc, "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           os.path.join(HERE, "csrc", "module.cu"), "-o", CUBIN + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed for k3moe_module.cubin")
    os.replace(CUBIN + ".tmp", CUBIN)
    return CUBIN


def build(force: bool = False, verbose: bool = False) -> str:
    nvcc = os.environ.get("NVCC", "nvcc")
    if not force and up_to_date():
        if not os.path.exists(CUBIN) or os.path.getmtime(CUBIN) < os.path.getmtime(OUT):
            build_cubin(nvcc)
        return OUT
    build_cubin(nvcc)
    cmd = [nvcc, *NVCC_FLAGS, SRC, "-o", OUT + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed for libk3moe.so")
    os.replace(OUT + ".tmp", OUT)
    with open(os.path.join(HERE, "ptxas.txt"), "w") as f:
        f.write(r.stderr)
    if verbose:
        sys.stderr.write(r.stderr)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
