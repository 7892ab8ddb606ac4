"""ctypes binding of the plain-C restatement (oracle/carl_oracle.c, built as
oracle/_ref/libcarloracle.so).  TEST INFRASTRUCTURE: tests only."""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_ref" / "libcarloracle.so"
_lib = None


class _Arena(ctypes.Structure):
    _fields_ = [("n_verts", ctypes.c_int), ("n_tris", ctypes.c_int), ("n_cells", ctypes.c_int),
                ("n_refs", ctypes.c_int), ("verts", ctypes.POINTER(ctypes.c_float)),
                ("tris", ctypes.POINTER(ctypes.c_int32)), ("prefix", ctypes.POINTER(ctypes.c_int32)),
                ("tri_idx", ctypes.POINTER(ctypes.c_int32))]


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "carl_oracle.c").stat().st_mtime:
            subprocess.run(["make", "-C", str(HERE), "port"], check=True, capture_output=True)
        lib = ctypes.CDLL(str(LIB))
        fp = ctypes.POINTER(ctypes.c_float)
        lib.co_arena_build.argtypes = [ctypes.c_char_p, ctypes.POINTER(_Arena)]
        lib.co_arena_free.argtypes = [ctypes.POINTER(_Arena)]
        lib.co_broadphase_cell.argtypes = [fp] * 5
        lib.co_broadphase_cell.restype = ctypes.c_int32
        lib.co_hash32.argtypes = [ctypes.c_uint32]
        lib.co_hash32.restype = ctypes.c_uint32
        lib.co_kickoff_row.argtypes = [ctypes.c_int32] * 3
        lib.co_kickoff_row.restype = ctypes.c_int32
        lib.co_kickoff_table.argtypes = [ctypes.c_void_p]
        _lib = lib
    return _lib


def arena(path) -> dict[str, np.ndarray]:
    lib = load()
    a = _Arena()
    if lib.co_arena_build(str(path).encode(), ctypes.byref(a)) != 0:
        raise RuntimeError(f"co_arena_build failed on {path}")
    out = {
        "verts": np.ctypeslib.as_array(a.verts, (a.n_verts * 3,)).reshape(-1, 3).copy(),
        "tris": np.ctypeslib.as_array(a.tris, (a.n_tris * 3,)).reshape(-1, 3).copy(),
        "prefix": np.ctypeslib.as_array(a.prefix, (a.n_cells + 1,)).copy(),
        "tri_idx": np.ctypeslib.as_array(a.tri_idx, (a.n_refs,)).copy(),
    }
    lib.co_arena_free(ctypes.byref(a))
    return out


def broadphase_cells(pos, vel, ang, cen, rot) -> np.ndarray:
    lib = load()
    f = lambda x, i: np.ascontiguousarray(x[i], dtype=np.float32).ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    return np.array([lib.co_broadphase_cell(f(pos, i), f(vel, i), f(ang, i), f(cen, i), f(rot, i))
                     for i in range(pos.shape[0])], dtype=np.int32)


def hash32(v: int) -> int:
    return load().co_hash32(v & 0xFFFFFFFF)


def kickoff_row(seed: int, sim: int, tick: int) -> int:
    return load().co_kickoff_row(seed, sim, tick)


def kickoff_table() -> np.ndarray:
    out = np.zeros((120, 4), dtype=np.int32)
    load().co_kickoff_table(out.ctypes.data)
    return out
