"""Minimal device-to-host / host-to-device copies of raw device pointers
through the CUDA runtime that torch loads (test infrastructure)."""

from __future__ import annotations

import ctypes
import glob
import os

import numpy as np
import torch

_rt = None


def _runtime():
    global _rt
    if _rt is None:
        base = os.path.join(os.path.dirname(torch.__file__), "..", "nvidia")
        cands = glob.glob(os.path.join(base, "cuda_runtime", "lib", "libcudart.so*")) + ["libcudart.so.12", "libcudart.so"]
        for c in cands:
            try:
                _rt = ctypes.CDLL(c)
                break
            except OSError:
                continue
        _rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    return _rt


def d2h(dst: np.ndarray, src_ptr: int) -> None:
    torch.cuda.synchronize()
    rc = _runtime().cudaMemcpy(dst.ctypes.data, src_ptr, dst.nbytes, 2)
    if rc != 0:
        raise RuntimeError(f"cudaMemcpy D2H failed ({rc})")


def h2d(dst_ptr: int, src: np.ndarray) -> None:
    rc = _runtime().cudaMemcpy(dst_ptr, np.ascontiguousarray(src).ctypes.data, src.nbytes, 1)
    if rc != 0:
        raise RuntimeError(f"cudaMemcpy H2D failed ({rc})")
