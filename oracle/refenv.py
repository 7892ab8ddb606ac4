"""Python wrappers of the reference oracles built under oracle/_ref/.

* RefCpu: the reference's physics compiled as host C++ (libcarlref_cpu.so).
* RefGpu: the reference's own CUDA build for sm_100a (libcarlref_cuda.so).

Both expose the snapshot field API of include/carlb.h so states can be moved
word for word between them and the product.  TEST INFRASTRUCTURE.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

from carl_b200 import capi

ROOT = Path(__file__).resolve().parents[1]
REF_DIR = ROOT / "oracle" / "_ref"
CPU_LIB = REF_DIR / "libcarlref_cpu.so"
GPU_LIB = REF_DIR / "libcarlref_cuda.so"
ARENA = REF_DIR / "arena.obj"

_libs: dict[str, ctypes.CDLL] = {}


def _arena_env() -> None:
    if "CARL_ARENA_OBJ" not in os.environ:
        for cand in (ARENA, ROOT / "carl_b200" / "_data" / "arena.obj"):
            if cand.exists():
                os.environ["CARL_ARENA_OBJ"] = str(cand)
                return


def _load(kind: str) -> ctypes.CDLL:
    if kind in _libs:
        return _libs[kind]
    _arena_env()
    path = CPU_LIB if kind == "cpu" else GPU_LIB
    if not path.exists():
        raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
    lib = ctypes.CDLL(str(path))
    p = "carlref_" if kind == "cpu" else "carlrefgpu_"
    vp, i32 = ctypes.c_void_p, ctypes.c_int32
    getattr(lib, p + "create").restype = vp
    getattr(lib, p + "create").argtypes = [i32] * 8
    getattr(lib, p + "error").restype = ctypes.c_char_p
    for name, args in [("destroy", [vp]), ("reset", [vp]), ("ticks", [vp, i32, vp, i32]),
                       ("env_step", [vp, i32, vp]), ("reset_dones", [vp]),
                       ("get_buffer", [vp, i32, vp]), ("read_field", [vp, i32, vp]),
                       ("write_field", [vp, i32, vp]), ("set_limits", [vp, i32, i32, i32, i32])]:
        getattr(lib, p + name).argtypes = args
    if kind == "cpu":
        lib.carlref_field_shape.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(i32)]
        lib.carlref_dims.argtypes = [vp, vp]
        lib.carlref_set_threads.argtypes = [i32]
        lib.carlref_repack.argtypes = [vp]
        lib.carlref_tick_partial.argtypes = [vp, i32, vp, i32]
        lib.carlref_arena_sizes.argtypes = [vp, vp]
        lib.carlref_arena_tables.argtypes = [vp] * 7
        lib.carlref_kickoff_table.argtypes = [vp]
    else:
        lib.carlrefgpu_tick_partial.argtypes = [vp, i32, vp, i32]
        lib.carlrefgpu_time_ticks.argtypes = [vp, i32, vp, i32, ctypes.POINTER(ctypes.c_float)]
        lib.carlrefgpu_apply_reset_state.argtypes = [vp, i32] + [vp] * 8 + [i32] + [vp] * 7
        lib.carlrefgpu_time_reset_steps.argtypes = ([vp, i32, vp, i32] + [vp] * 12
                                                    + [ctypes.POINTER(ctypes.c_float)] * 2)
    _libs[kind] = lib
    return lib


def _addr(a):
    return None if a is None else a.ctypes.data


class _RefEnv:
    kind = "cpu"
    prefix = "carlref_"

    def __init__(self, n_sim, n_blue, n_orange, seed=0, frameskip=1, invert_orange=True, normalize=False,
                 previous_controls=False):
        self.lib = _load(self.kind)
        h = getattr(self.lib, self.prefix + "create")(n_sim, n_blue, n_orange, seed, frameskip,
                                                      int(invert_orange), int(normalize), int(previous_controls))
        if not h:
            raise RuntimeError(getattr(self.lib, self.prefix + "error")().decode())
        self.h = ctypes.c_void_p(h)
        self.n_sim, self.n_cars = n_sim, n_blue + n_orange
        self.n_blue, self.n_orange = n_blue, n_orange
        self.obs_dim = 9 + self.n_cars * 21 + 68 + 6 + (self.n_cars - 1) * 6 + 6 + 2 + 5 + (8 if previous_controls else 0)
        self.state_dim = 9 + self.n_cars * 22 + 34

    def _call(self, name, *args):
        st = getattr(self.lib, self.prefix + name)(self.h, *args)
        if st != 0:
            raise RuntimeError(getattr(self.lib, self.prefix + "error")().decode())

    def close(self):
        if self.h:
            getattr(self.lib, self.prefix + "destroy")(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def field_shape(self, name: str):
        n, ns = self.n_sim * self.n_cars, self.n_sim
        width = {"CAR_POS": 3, "CAR_VEL": 3, "CAR_ANG": 3, "CAR_ROT": 4, "CAR_CEN": 3, "CAR_IMP": 3,
                 "CAR_WHEEL_SOURCE": 4, "CAR_WHEEL_CONTACT": 4, "CAR_CONTROLS": 8, "CAR_INTERNAL": 24,
                 "SUSP_SCALARS": 15, "SUSP_RAY_DIST": 4, "SUSP_RAY_NORMAL": 12, "SUSP_LAT_FRICTION": 4,
                 "SUSP_LON_FRICTION": 4, "MAN_NORMAL0": 3, "BALL_POS": 3, "BALL_VEL": 3, "BALL_ANG": 3,
                 "BALL_IMP": 3, "BALL_INT_POS": 3, "BALL_INT_VEL": 3, "BALL_EXP_POS": 3, "BALL_EXP_VEL": 3,
                 "GOALS": 5, "PAD_COOLDOWNS": 34, "DIAG_SAT_PAIRS": 33,
                 "DIAG_CC_COUNT": max(1, self.n_cars * (self.n_cars - 1) // 2)}.get(name, 1)
        if name == "TICK_COUNT":
            return 1, 1
        sim_fields = {"BALL_POS", "BALL_VEL", "BALL_ANG", "BALL_IMP", "BALL_INT_POS", "BALL_INT_VEL",
                      "BALL_EXP_POS", "BALL_EXP_VEL", "BALL_INT_VALID", "EPISODE_TICKS", "LAST_TOUCH_TICKS",
                      "BALL_ARENA_CONTACT_TICK", "GOALS", "PAD_COOLDOWNS", "DIAG_CC_COUNT"}
        return (ns if name in sim_fields else n), width

    def read_field(self, name: str) -> np.ndarray:
        rows, width = self.field_shape(name)
        out = np.zeros((rows, width), dtype=np.uint32)
        self._call("read_field", capi.FIELD[name], out.ctypes.data)
        return out

    def write_field(self, name: str, words: np.ndarray) -> None:
        rows, width = self.field_shape(name)
        arr = np.ascontiguousarray(words).view(np.uint32).reshape(rows, width)
        self._call("write_field", capi.FIELD[name], arr.ctypes.data)

    def snapshot(self):
        return {name: self.read_field(name) for name in capi.PERSISTENT_FIELDS}

    def restore(self, snap):
        for name, words in snap.items():
            self.write_field(name, words)

    def ticks(self, kind: int, actions: np.ndarray, n_ticks: int) -> None:
        self._call("ticks", kind, np.ascontiguousarray(actions).ctypes.data, n_ticks)

    def tick_partial(self, kind: int, actions: np.ndarray, last_stage: int) -> None:
        """One tick, stopping after stage `last_stage` (0..11)."""
        self._call("tick_partial", kind, np.ascontiguousarray(actions).ctypes.data, last_stage)

    def env_step(self, kind: int, actions: np.ndarray) -> None:
        self._call("env_step", kind, np.ascontiguousarray(actions).ctypes.data)

    def reset(self):
        self._call("reset")

    def reset_dones(self):
        self._call("reset_dones")

    def set_limits(self, max_ticks=-1, overtime=-1, no_touch=-1, frameskip=-1):
        self._call("set_limits", max_ticks, overtime, no_touch, frameskip)

    def get_buffer(self, which: int) -> np.ndarray:
        ns, nc = self.n_sim, self.n_cars
        spec = {capi.BUF_OBS: ((ns, nc, self.obs_dim), np.float32),
                capi.BUF_TRANSITION_OBS: ((ns, nc, self.obs_dim), np.float32),
                capi.BUF_STATE: ((ns, self.state_dim), np.float32),
                capi.BUF_TRANSITION_STATE: ((ns, self.state_dim), np.float32),
                capi.BUF_REWARDS: ((ns,), np.float32), capi.BUF_DONES: ((ns,), np.uint8),
                capi.BUF_SCORE_DIFFERENCE: ((ns,), np.int32), capi.BUF_EPISODE_TICKS: ((ns,), np.int32),
                capi.BUF_TRANSITION_SCORE_DIFFERENCE: ((ns,), np.int32),
                capi.BUF_TRANSITION_EPISODE_TICKS: ((ns,), np.int32),
                capi.BUF_OVERTIME: ((ns,), np.uint8), capi.BUF_TRANSITION_OVERTIME: ((ns,), np.uint8)}[which]
        out = np.zeros(spec[0], dtype=spec[1])
        self._call("get_buffer", which, out.ctypes.data)
        return out


class RefCpu(_RefEnv):
    kind = "cpu"
    prefix = "carlref_"

    @staticmethod
    def set_threads(n: int) -> int:
        return _load("cpu").carlref_set_threads(n)

    def repack(self):
        self._call("repack")


class RefGpu(_RefEnv):
    kind = "gpu"
    prefix = "carlrefgpu_"

    def time_ticks(self, kind: int, actions: np.ndarray, n_ticks: int) -> float:
        ms = ctypes.c_float()
        self._call("time_ticks", kind, np.ascontiguousarray(actions).ctypes.data, n_ticks, ctypes.byref(ms))
        return ms.value

    def time_reset_steps(self, kind: int, actions: np.ndarray, n_steps: int, reset: dict | None = None,
                         masks: np.ndarray | None = None) -> tuple[float, float]:
        """Device ms of n_steps env steps and of the masked resets after each
        (reset: one row per sim of every apply_reset_state input, demoed u8;
        masks [n_steps, n_sim]); without masks the steps run alone."""
        step_ms, reset_ms = ctypes.c_float(), ctypes.c_float()
        order = ["ball_position", "ball_velocity", "ball_angular_velocity", "car_position", "car_rotation",
                 "car_velocity", "car_angular_velocity", "car_demoed", "blue_score", "orange_score", "episode_ticks"]
        arrs = [None if reset is None else np.ascontiguousarray(reset[o]) for o in order]
        masks = None if masks is None else np.ascontiguousarray(masks, dtype=np.uint8)
        actions = np.ascontiguousarray(actions)
        self._call("time_reset_steps", kind, actions.ctypes.data, n_steps, *[_addr(a) for a in arrs],
                   _addr(masks), ctypes.byref(step_ms), ctypes.byref(reset_ms))
        return step_ms.value, reset_ms.value

    def apply_reset_state(self, n_selected, ball_position, ball_velocity, ball_angular_velocity, car_position,
                          car_rotation, car_velocity, car_angular_velocity, car_demoed, demoed_is_byte,
                          car_boost=None, car_internal_state=None, blue_score=None, orange_score=None,
                          episode_ticks=None, simulation_indices=None, reset_mask=None):
        arrs = [ball_position, ball_velocity, ball_angular_velocity, car_position, car_rotation, car_velocity,
                car_angular_velocity, car_demoed]
        self._call("apply_reset_state", n_selected, *[_addr(a) for a in arrs], int(demoed_is_byte),
                   _addr(car_boost), _addr(car_internal_state), _addr(blue_score), _addr(orange_score),
                   _addr(episode_ticks), _addr(simulation_indices), _addr(reset_mask))


def reference_arena_tables(ref: RefCpu) -> dict[str, np.ndarray]:
    """The reference's arena tables (src/ArenaMesh.cu:15-125) from a RefCpu env."""
    lib = _load("cpu")
    sizes = np.zeros(4, dtype=np.int32)
    lib.carlref_arena_sizes(ref.h, sizes.ctypes.data)
    nv, nt, nc, nr = (int(x) for x in sizes)
    out = {"verts": np.zeros((nv, 3), np.float32), "tris": np.zeros((nt, 3), np.int32),
           "prefix": np.zeros(nc + 1, np.int32), "tri_idx": np.zeros(nr, np.int32),
           "edge_angles": np.zeros((nt, 3), np.float32), "ball_tri_idx": np.zeros(nr, np.int32)}
    lib.carlref_arena_tables(ref.h, *[out[k].ctypes.data for k in
                                      ("verts", "tris", "prefix", "tri_idx", "edge_angles", "ball_tri_idx")])
    return out


def reference_kickoff_table() -> np.ndarray:
    out = np.zeros((120, 4), dtype=np.int32)
    _load("cpu").carlref_kickoff_table(out.ctypes.data)
    return out
