"""Launch the reference's own kernels (built from its sources for sm_100a into
oracle/_ref by oracle/Makefile) through the CUDA driver API — test
infrastructure: these are the GPU oracle for the bit-exact stages."""
from __future__ import annotations

import ctypes
import os

import torch

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")

_cuda = None
_modules = {}


def _drv():
    global _cuda
    if _cuda is None:
        _cuda = ctypes.CDLL("libcuda.so.1")
        _cuda.cuModuleLoad.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]
        _cuda.cuModuleGetFunction.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
        _cuda.cuLaunchKernel.argtypes = [ctypes.c_void_p] + [ctypes.c_uint] * 6 + [ctypes.c_uint, ctypes.c_void_p,
                                                                                  ctypes.POINTER(ctypes.c_void_p),
                                                                                  ctypes.c_void_p]
        _cuda.cuLaunchCooperativeKernel.argtypes = [ctypes.c_void_p] + [ctypes.c_uint] * 6 + [
            ctypes.c_uint, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
    return _cuda


def available(module: str) -> bool:
    return os.path.exists(os.path.join(REF_DIR, module + ".cubin"))


def function(module: str, entry: str):
    """`module`: a cubin name under oracle/_ref, or a path ending in .cubin."""
    torch.cuda.init()
    torch.zeros(1, device="cuda")  # the primary context is current
    d = _drv()
    if module not in _modules:
        m = ctypes.c_void_p()
        path = module if module.endswith(".cubin") else os.path.join(REF_DIR, module + ".cubin")
        rc = d.cuModuleLoad(ctypes.byref(m), path.encode())
        if rc != 0:
            raise RuntimeError(f"cuModuleLoad({module}) = {rc}")
        _modules[module] = m
    f = ctypes.c_void_p()
    rc = d.cuModuleGetFunction(ctypes.byref(f), _modules[module], entry.encode())
    if rc != 0:
        raise RuntimeError(f"cuModuleGetFunction({entry}) = {rc}")
    return f


def allow_smem(f, nbytes: int):
    """Let `f` launch with `nbytes` of dynamic shared memory (CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES)."""
    d = _drv()
    d.cuFuncSetAttribute.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    rc = d.cuFuncSetAttribute(f, 8, int(nbytes))
    if rc != 0:
        raise RuntimeError(f"cuFuncSetAttribute = {rc}")


def launch(f, grid, block, args, smem=0):
    """args: ctypes values (c_void_p for device pointers, c_int for ints)."""
    holders = [ctypes.pointer(a) for a in args]
    arr = (ctypes.c_void_p * len(args))(*[ctypes.cast(h, ctypes.c_void_p) for h in holders])
    s = torch.cuda.current_stream().cuda_stream
    rc = _drv().cuLaunchKernel(f, grid[0], grid[1], grid[2], block[0], block[1], block[2], smem, s, arr, None)
    if rc != 0:
        raise RuntimeError(f"cuLaunchKernel = {rc}")


def launch_cooperative(f, grid, block, args, smem=0):
    """launch() as a cooperative launch: the driver starts every block at once or refuses the launch, so a
    kernel whose blocks wait on one another (a grid barrier) cannot wait for a block that never starts."""
    holders = [ctypes.pointer(a) for a in args]
    arr = (ctypes.c_void_p * len(args))(*[ctypes.cast(h, ctypes.c_void_p) for h in holders])
    s = torch.cuda.current_stream().cuda_stream
    rc = _drv().cuLaunchCooperativeKernel(f, grid[0], grid[1], grid[2], block[0], block[1], block[2], smem, s, arr)
    if rc != 0:
        raise RuntimeError(f"cuLaunchCooperativeKernel = {rc}")


def P(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def I(v: int):
    return ctypes.c_int(int(v))
