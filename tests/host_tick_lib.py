"""ctypes wrapper of tests/host_tick (the product's physics compiled for the
host, stepped serially in the kernel's stage order).  TEST INFRASTRUCTURE."""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

from carl_b200 import capi

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "host_tick" / "host_tick.cpp"
KA = ROOT / "tests" / "host_tick" / "known_answers.cpp"
LIB = ROOT / "tests" / "host_tick" / "_build" / "libhosttick.so"
DEPS = [SRC, KA, ROOT / "tests" / "host_tick" / "host_intrinsics.h", *sorted((ROOT / "carl_b200" / "csrc").glob("*.cuh")), *sorted((ROOT / "carl_b200" / "csrc").glob("*.hpp")),
        ROOT / "carl_b200" / "csrc" / "arena.cpp", ROOT / "carl_b200" / "csrc" / "tables.cpp"]
_lib = None


def build() -> Path:
    if not LIB.exists() or any(d.stat().st_mtime > LIB.stat().st_mtime for d in DEPS):
        LIB.parent.mkdir(exist_ok=True)
        subprocess.run(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-include", "algorithm",
                        "-o", str(LIB), str(SRC), str(KA), str(ROOT / "carl_b200/csrc/arena.cpp"),
                        str(ROOT / "carl_b200/csrc/tables.cpp")], check=True)
    return LIB


def lib():
    """The host build library (for the known-answer functions)."""
    return _load()


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        lib.hosttick_create.restype = ctypes.c_void_p
        lib.hosttick_create.argtypes = [ctypes.c_char_p] + [ctypes.c_int] * 4
        lib.hosttick_error.restype = ctypes.c_char_p
        lib.hosttick_destroy.argtypes = [ctypes.c_void_p]
        lib.hosttick_read_field.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        lib.hosttick_write_field.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        lib.hosttick_ticks.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        lib.hosttick_arena_sizes.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.hosttick_arena_tables.argtypes = [ctypes.c_void_p] * 8
        lib.hosttick_kickoff_table.argtypes = [ctypes.c_void_p] * 2
        lib.hosttick_ball_grid.argtypes = [ctypes.c_void_p] * 3
        lib.hosttick_ball_lists.argtypes = [ctypes.c_void_p] * 3
        lib.hosttick_load_metadata.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
        _lib = lib
    return _lib


class HostTick:
    def __init__(self, arena_path: str, n_sim: int, n_blue: int, n_orange: int, seed: int = 0):
        self.lib = _load()
        h = self.lib.hosttick_create(str(arena_path).encode(), n_sim, n_blue, n_orange, seed)
        if not h:
            raise RuntimeError(self.lib.hosttick_error().decode())
        self.h = ctypes.c_void_p(h)
        self.n_sim, self.n_cars = n_sim, n_blue + n_orange

    def close(self):
        if self.h:
            self.lib.hosttick_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def field_shape(self, name):
        from oracle.refenv import _RefEnv
        return _RefEnv.field_shape(self, name)

    def read_field(self, name):
        rows, width = self.field_shape(name)
        out = np.zeros((rows, width), dtype=np.uint32)
        assert self.lib.hosttick_read_field(self.h, capi.FIELD[name], out.ctypes.data) == 0
        return out

    def write_field(self, name, words):
        rows, width = self.field_shape(name)
        arr = np.ascontiguousarray(words).view(np.uint32).reshape(rows, width)
        assert self.lib.hosttick_write_field(self.h, capi.FIELD[name], arr.ctypes.data) == 0

    def snapshot(self):
        return {n: self.read_field(n) for n in capi.PERSISTENT_FIELDS}

    def restore(self, snap):
        for n, w in snap.items():
            self.write_field(n, w)

    def arena_tables(self) -> dict[str, np.ndarray]:
        """The product's arena tables (carl_b200/csrc/arena.cpp)."""
        sizes = np.zeros(4, dtype=np.int32)
        self.lib.hosttick_arena_sizes(self.h, sizes.ctypes.data)
        nv, nt, nc, nr = (int(x) for x in sizes)
        out = {"verts": np.zeros((nv, 3), np.float32), "tris": np.zeros((nt, 3), np.int32),
               "prefix": np.zeros(nc + 1, np.int32), "tri_idx": np.zeros(nr, np.int32),
               "edge_angles": np.zeros((nt, 3), np.float32), "normals": np.zeros((nt, 3), np.float32),
               "flags": np.zeros(nt, np.int32)}
        self.lib.hosttick_arena_tables(self.h, *[out[k].ctypes.data for k in
                                                 ("verts", "tris", "prefix", "tri_idx", "edge_angles", "normals",
                                                  "flags")])
        return out

    def load_metadata(self, path) -> None:
        """Native mesh metadata into the product's arena tables (raises with its error)."""
        if self.lib.hosttick_load_metadata(self.h, str(path).encode()) != 0:
            raise RuntimeError(self.lib.hosttick_error().decode())

    def ball_grid(self):
        """(origin[3], cell size, dims[3], cell starts, cell triangle lists) of the product's ball grid."""
        geom = np.zeros(4, np.float32)
        dims = np.zeros(4, np.int32)
        self.lib.hosttick_ball_grid(self.h, geom.ctypes.data, dims.ctypes.data)
        n = int(dims[0]) * int(dims[1]) * int(dims[2])
        start = np.zeros(n + 1, np.int32)
        tris = np.zeros(max(1, int(dims[3])), np.int32)
        self.lib.hosttick_ball_lists(self.h, start.ctypes.data, tris.ctypes.data)
        return geom[:3], float(geom[3]), dims[:3], start, tris

    def kickoff_table(self) -> np.ndarray:
        out = np.zeros((120, 4), dtype=np.int32)
        self.lib.hosttick_kickoff_table(self.h, out.ctypes.data)
        return out

    def ticks(self, controls: np.ndarray, n: int):
        self.lib.hosttick_ticks(self.h, np.ascontiguousarray(controls).ctypes.data, n)
