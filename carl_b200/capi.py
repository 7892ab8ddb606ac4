"""ctypes binding of the C ABI in include/carlb.h (libcarlb.so).

This is the thin host layer the Python front end, the tests and the benchmark
use.  It never falls back to anything: if the native library is missing or was
built for another GPU, creating an env raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent
_LIB_PATH = _PKG / "libcarlb.so"
_lib = None

# ---- enums of carlb.h -------------------------------------------------------
OK, ERR_VALUE, ERR_TYPE, ERR_CUDA, ERR_STATE = range(5)
ACTIONS_DISCRETE, ACTIONS_CONTINUOUS, ACTIONS_DIRECT = range(3)
(BUF_OBS, BUF_TRANSITION_OBS, BUF_STATE, BUF_TRANSITION_STATE, BUF_REWARDS, BUF_DONES,
 BUF_SCORE_DIFFERENCE, BUF_EPISODE_TICKS, BUF_TRANSITION_SCORE_DIFFERENCE,
 BUF_TRANSITION_EPISODE_TICKS, BUF_OVERTIME, BUF_TRANSITION_OVERTIME) = range(12)
DT_F32, DT_I32, DT_BOOL, DT_I64 = range(4)
SOURCE_LAGGED_LATERAL_FRICTION = 1  # compat_flags bit; 0 = the reference CUDA build's semantics
LIMIT_MAX_TICKS, LIMIT_OVERTIME_TIMEOUT_TICKS, LIMIT_NO_TOUCH_TIMEOUT_TICKS, LIMIT_FRAMESKIP = range(4)

FIELDS = [
    "CAR_POS", "CAR_VEL", "CAR_ANG", "CAR_ROT", "CAR_CEN", "CAR_IMP", "CAR_IS_DEMOED",
    "CAR_DEMO_TIMER", "CAR_CONTACT_IDX", "CAR_CONTACT_COOLDOWN", "CAR_BALL_HIT_TICK",
    "CAR_BALL_CONTACT_TICK", "CAR_WHEEL_SOURCE", "CAR_WHEEL_CONTACT", "CAR_ARENA_CONTACT_TICK",
    "CAR_CONTROLS", "CAR_INTERNAL", "SUSP_SCALARS", "SUSP_RAY_DIST", "SUSP_RAY_NORMAL",
    "SUSP_LAT_FRICTION", "SUSP_LON_FRICTION", "MAN_COUNT", "MAN_NORMAL0", "BALL_POS", "BALL_VEL",
    "BALL_ANG", "BALL_IMP", "BALL_INT_POS", "BALL_INT_VEL", "BALL_EXP_POS", "BALL_EXP_VEL",
    "BALL_INT_VALID", "EPISODE_TICKS", "LAST_TOUCH_TICKS", "BALL_ARENA_CONTACT_TICK", "GOALS",
    "PAD_COOLDOWNS", "TICK_COUNT", "DIAG_CELL_IDX", "DIAG_NUM_TRIS", "DIAG_SAT_PAIRS", "DIAG_CC_COUNT",
]
FIELD = {name: i for i, name in enumerate(FIELDS)}
PERSISTENT_FIELDS = FIELDS[: FIELD["TICK_COUNT"] + 1]
DIAG_FIELDS = FIELDS[FIELD["DIAG_CELL_IDX"]:]

# Word kinds: 'f' float32, 'i' int32.  Mixed records list one letter per word.
FIELD_KINDS = {
    "CAR_IS_DEMOED": "i", "CAR_CONTACT_IDX": "i", "CAR_BALL_HIT_TICK": "i", "CAR_BALL_CONTACT_TICK": "i",
    "CAR_WHEEL_SOURCE": "i", "CAR_WHEEL_CONTACT": "i", "CAR_ARENA_CONTACT_TICK": "i",
    "CAR_CONTROLS": "fffffiii", "CAR_INTERNAL": "ifffiifiiiififffffiiifff",
    "MAN_COUNT": "i", "BALL_INT_VALID": "i", "EPISODE_TICKS": "i", "LAST_TOUCH_TICKS": "i",
    "BALL_ARENA_CONTACT_TICK": "i", "GOALS": "i", "TICK_COUNT": "i", "DIAG_CELL_IDX": "i",
    "DIAG_NUM_TRIS": "i", "DIAG_SAT_PAIRS": "i", "DIAG_CC_COUNT": "i",
}


def field_kinds(name: str, width: int) -> str:
    """One 'f'/'i' letter per word of `name`."""
    k = FIELD_KINDS.get(name, "f")
    return k * width if len(k) == 1 else k


class Config(ctypes.Structure):
    _fields_ = [
        ("n_sim", ctypes.c_int32), ("n_blue", ctypes.c_int32), ("n_orange", ctypes.c_int32),
        ("seed", ctypes.c_int32), ("frameskip", ctypes.c_int32), ("invert_orange", ctypes.c_int32),
        ("normalize", ctypes.c_int32), ("previous_controls", ctypes.c_int32), ("device", ctypes.c_int32),
        ("compat_flags", ctypes.c_int32), ("sim_offset", ctypes.c_int64),
    ]


class CarlbError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def library_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Loads libcarlb.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        raise ImportError(f"{_LIB_PATH} is missing: build it with carl_b200._build.build()")
    if "CARL_ARENA_OBJ" not in os.environ:
        data = _PKG / "_data" / "arena.obj"
        if data.exists():
            os.environ["CARL_ARENA_OBJ"] = str(data)
    lib = ctypes.CDLL(str(_LIB_PATH))
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    lib.carlb_create.argtypes = [ctypes.POINTER(Config), ctypes.POINTER(vp)]
    lib.carlb_destroy.argtypes = [vp]
    lib.carlb_last_error.argtypes = [vp]
    lib.carlb_last_error.restype = ctypes.c_char_p
    lib.carlb_env_step.argtypes = [vp, i32, vp]
    lib.carlb_ticks.argtypes = [vp, i32, vp, i32]
    lib.carlb_ticks_host.argtypes = [vp, i32, vp, i32, vp]
    lib.carlb_ticks_static_scratch.argtypes = [vp, i32, vp, i32]
    lib.carlb_reset.argtypes = [vp]
    lib.carlb_reset_dones.argtypes = [vp]
    lib.carlb_apply_reset_state.argtypes = [vp, i32] + [vp] * 8 + [i32] + [vp] * 7
    lib.carlb_set_ball.argtypes = [vp, i32, vp, vp, vp, vp]
    lib.carlb_set_car.argtypes = [vp, i32, vp, vp, vp, vp, vp, i32, vp, vp, vp]
    lib.carlb_set_match_state.argtypes = [vp, i32, vp, vp, vp, vp]
    lib.carlb_reset_boost_pads.argtypes = [vp, i32, vp]
    lib.carlb_get_buffer.argtypes = [vp, i32, ctypes.POINTER(vp), ctypes.POINTER(i64), ctypes.POINTER(i32), ctypes.POINTER(i32)]
    lib.carlb_set_limit.argtypes = [vp, i32, i32]
    lib.carlb_get_limit.argtypes = [vp, i32, ctypes.POINTER(i32)]
    lib.carlb_dims.argtypes = [vp, ctypes.POINTER(i32)]
    lib.carlb_stream.argtypes = [vp]
    lib.carlb_stream.restype = vp
    lib.carlb_synchronize.argtypes = [vp]
    lib.carlb_field_shape.argtypes = [vp, i32, ctypes.POINTER(i64), ctypes.POINTER(i32)]
    lib.carlb_read_field.argtypes = [vp, i32, vp]
    lib.carlb_write_field.argtypes = [vp, i32, vp]
    lib.carlb_set_diagnostics.argtypes = [vp, i32]
    lib.carlb_last_tick_ms.argtypes = [vp, ctypes.POINTER(ctypes.c_float)]
    lib.carlb_set_stage_timing.argtypes = [vp, i32]
    lib.carlb_stage_times.argtypes = [vp, ctypes.POINTER(ctypes.c_float), i32, ctypes.POINTER(i32)]
    lib.carlb_stage_work.argtypes = [vp, ctypes.POINTER(i32)]
    lib.carlb_action_mask.argtypes = [vp, i64, i32, i32, vp, vp]
    _lib = lib
    return lib


def _ptr(x) -> int | None:
    """Device/host address of a torch tensor, numpy array, int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    return x.data_ptr()


def action_mask(obs, rows: int, obs_dim: int, previous_controls: bool, mask, stream: int) -> None:
    """carlb_action_mask: uint8 [rows, 18] action mask of float32 [rows, obs_dim]
    observation rows (device addresses or tensors), enqueued on `stream`."""
    lib = load()
    st = lib.carlb_action_mask(_ptr(obs), rows, obs_dim, int(previous_controls), _ptr(mask), stream)
    if st != OK:
        raise CarlbError(st, lib.carlb_last_error(None).decode())


class Env:
    """One env on one GPU (owns device state, outputs and a CUDA stream)."""

    def __init__(self, n_sim: int, n_blue: int, n_orange: int, seed: int = 0, frameskip: int = 1,
                 invert_orange: bool = True, normalize: bool = False, previous_controls: bool = False,
                 device: int = 0, sim_offset: int = 0, compat_flags: int = 0):
        self._lib = load()
        cfg = Config(n_sim, n_blue, n_orange, seed, frameskip, int(invert_orange), int(normalize),
                     int(previous_controls), device, compat_flags, sim_offset)
        h = ctypes.c_void_p()
        st = self._lib.carlb_create(ctypes.byref(cfg), ctypes.byref(h))
        if st != OK:
            raise CarlbError(st, self._lib.carlb_last_error(None).decode())
        self._h = h
        dims = (ctypes.c_int32 * 5)()
        self._lib.carlb_dims(self._h, dims)
        self.n_sim, self.n_cars, self.obs_dim, self.act_dim, self.state_dim = list(dims)
        self.device = device
        self._ext_stream = None
        self._pending: list = []

    def _order_after_torch(self, *inputs) -> list:
        """Orders the env stream after the producer of torch CUDA inputs.

        Device inputs are read on the env's own (non-blocking) stream; a torch
        tensor may still be being written on torch's current stream, so the env
        stream waits for it, as the reference's DLPack handoff
        (``__dlpack__(stream=env_stream)``) does.  Returns the torch inputs, which
        `_keep_until_read` holds until the env stream has passed the call."""
        tensors = [x for x in inputs if x is not None and getattr(x, "is_cuda", False)]
        if tensors:
            import torch

            if self._ext_stream is None:
                self._ext_stream = torch.cuda.ExternalStream(self.stream, device=tensors[0].device)
            self._ext_stream.wait_stream(torch.cuda.current_stream(tensors[0].device))
        return tensors

    def _keep_until_read(self, tensors: list) -> None:
        """Keeps torch inputs alive (so torch's caching allocator cannot hand
        their memory to new tensors) until an event recorded on the env stream
        after the reads has completed, like the reference's pending-reset
        capsules (python/carl.cu:613-629)."""
        import torch

        while self._pending and self._pending[0][0].query():
            self._pending.pop(0)
        if tensors:
            ev = torch.cuda.Event()
            ev.record(self._ext_stream)
            self._pending.append((ev, tensors))

    def _check(self, st: int) -> None:
        if st != OK:
            raise CarlbError(st, self._lib.carlb_last_error(self._h).decode())

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.carlb_synchronize(self._h)
            self._pending = []
            self._ext_stream = None
            self._lib.carlb_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- stepping ----
    def ticks(self, kind: int, actions, n_ticks: int) -> None:
        keep = self._order_after_torch(actions)
        self._check(self._lib.carlb_ticks(self._h, kind, _ptr(actions), n_ticks))
        self._keep_until_read(keep)

    def ticks_static_scratch(self, kind: int, actions, n_ticks: int) -> None:
        """carlb_ticks with the fixed-size static stage scratch (allocates nothing)."""
        keep = self._order_after_torch(actions)
        self._check(self._lib.carlb_ticks_static_scratch(self._h, kind, _ptr(actions), n_ticks))
        self._keep_until_read(keep)

    def ticks_host(self, kind: int, host_actions: np.ndarray, n_ticks: int, host_rewards: np.ndarray | None = None) -> None:
        self._check(self._lib.carlb_ticks_host(self._h, kind, _ptr(host_actions), n_ticks, _ptr(host_rewards)))

    def env_step(self, kind: int, actions) -> None:
        keep = self._order_after_torch(actions)
        self._check(self._lib.carlb_env_step(self._h, kind, _ptr(actions)))
        self._keep_until_read(keep)

    def reset(self) -> None:
        self._check(self._lib.carlb_reset(self._h))

    def reset_dones(self) -> None:
        self._check(self._lib.carlb_reset_dones(self._h))

    def apply_reset_state(self, n_selected, ball_position, ball_velocity, ball_angular_velocity, car_position,
                          car_rotation, car_velocity, car_angular_velocity, car_demoed, demoed_is_byte,
                          car_boost=None, car_internal_state=None, blue_score=None, orange_score=None,
                          episode_ticks=None, simulation_indices=None, reset_mask=None) -> None:
        args = [ball_position, ball_velocity, ball_angular_velocity, car_position, car_rotation, car_velocity,
                car_angular_velocity, car_demoed]
        keep = self._order_after_torch(*args, car_boost, car_internal_state, blue_score, orange_score,
                                       episode_ticks, simulation_indices, reset_mask)
        self._check(self._lib.carlb_apply_reset_state(
            self._h, n_selected, *[_ptr(a) for a in args], int(demoed_is_byte), _ptr(car_boost),
            _ptr(car_internal_state), _ptr(blue_score), _ptr(orange_score), _ptr(episode_ticks),
            _ptr(simulation_indices), _ptr(reset_mask)))
        self._keep_until_read(keep)

    def set_ball(self, n, pos, vel, ang, indices=None) -> None:
        keep = self._order_after_torch(pos, vel, ang, indices)
        self._check(self._lib.carlb_set_ball(self._h, n, _ptr(pos), _ptr(vel), _ptr(ang), _ptr(indices)))
        self._keep_until_read(keep)

    def set_car(self, n, pos, rot, vel, ang, demoed, demoed_is_byte, boost=None, internal=None, indices=None) -> None:
        keep = self._order_after_torch(pos, rot, vel, ang, demoed, boost, internal, indices)
        self._check(self._lib.carlb_set_car(self._h, n, _ptr(pos), _ptr(rot), _ptr(vel), _ptr(ang), _ptr(demoed),
                                            int(demoed_is_byte), _ptr(boost), _ptr(internal), _ptr(indices)))
        self._keep_until_read(keep)

    def set_match_state(self, n, blue, orange, ticks, indices=None) -> None:
        keep = self._order_after_torch(blue, orange, ticks, indices)
        self._check(self._lib.carlb_set_match_state(self._h, n, _ptr(blue), _ptr(orange), _ptr(ticks), _ptr(indices)))
        self._keep_until_read(keep)

    def reset_boost_pads(self, n, indices=None) -> None:
        keep = self._order_after_torch(indices)
        self._check(self._lib.carlb_reset_boost_pads(self._h, n, _ptr(indices)))
        self._keep_until_read(keep)

    # ---- outputs / properties ----
    def buffer(self, which: int):
        """(device pointer, shape tuple, carlb dtype) of an output buffer."""
        data = ctypes.c_void_p()
        shape = (ctypes.c_int64 * 3)()
        ndim = ctypes.c_int32()
        dt = ctypes.c_int32()
        self._check(self._lib.carlb_get_buffer(self._h, which, ctypes.byref(data), shape, ctypes.byref(ndim), ctypes.byref(dt)))
        return data.value, tuple(shape[: ndim.value]), dt.value

    def set_limit(self, which: int, value: int) -> None:
        self._check(self._lib.carlb_set_limit(self._h, which, value))

    def get_limit(self, which: int) -> int:
        v = ctypes.c_int32()
        self._check(self._lib.carlb_get_limit(self._h, which, ctypes.byref(v)))
        return v.value

    @property
    def stream(self) -> int:
        return self._lib.carlb_stream(self._h) or 0

    def synchronize(self) -> None:
        self._check(self._lib.carlb_synchronize(self._h))

    def set_diagnostics(self, enabled: bool) -> None:
        self._check(self._lib.carlb_set_diagnostics(self._h, int(enabled)))

    def last_tick_ms(self) -> float:
        ms = ctypes.c_float()
        self._check(self._lib.carlb_last_tick_ms(self._h, ctypes.byref(ms)))
        return ms.value

    STAGES = ["ballPrep", "flat", "ray", "ctlSusp", "contact", "carCar", "ball", "finish"]

    def set_stage_timing(self, enabled: bool) -> None:
        self._check(self._lib.carlb_set_stage_timing(self._h, int(enabled)))

    def stage_times(self) -> dict[str, float]:
        """Milliseconds per stage kernel of the last timed tick (staged path)."""
        ms = (ctypes.c_float * 16)()
        n = ctypes.c_int32()
        self._check(self._lib.carlb_stage_times(self._h, ms, 16, ctypes.byref(n)))
        return {self.STAGES[k]: ms[k] for k in range(n.value)}

    STAGE_WORK = ("plane_cars", "sat_cars", "moving_balls", "car_car_sims")

    def stage_work(self) -> dict[str, int]:
        """Work-list sizes of the last tick of the last launch (all sim slices)."""
        counts = (ctypes.c_int32 * 4)()
        self._check(self._lib.carlb_stage_work(self._h, counts))
        return {name: int(counts[k]) for k, name in enumerate(self.STAGE_WORK)}

    # ---- snapshot ----
    def field_shape(self, name: str) -> tuple[int, int]:
        rows, width = ctypes.c_int64(), ctypes.c_int32()
        self._check(self._lib.carlb_field_shape(self._h, FIELD[name], ctypes.byref(rows), ctypes.byref(width)))
        return rows.value, width.value

    def read_field(self, name: str) -> np.ndarray:
        """Raw 32-bit words, shape [rows, width] (view as float32/int32 per FIELD_KINDS)."""
        rows, width = self.field_shape(name)
        out = np.zeros((rows, width), dtype=np.uint32)
        self._check(self._lib.carlb_read_field(self._h, FIELD[name], out.ctypes.data))
        return out

    def write_field(self, name: str, words: np.ndarray) -> None:
        rows, width = self.field_shape(name)
        arr = np.ascontiguousarray(words).view(np.uint32).reshape(rows, width)
        self._check(self._lib.carlb_write_field(self._h, FIELD[name], arr.ctypes.data))

    def snapshot(self) -> dict[str, np.ndarray]:
        return {name: self.read_field(name) for name in PERSISTENT_FIELDS}

    def restore(self, snap: dict[str, np.ndarray]) -> None:
        for name, words in snap.items():
            self.write_field(name, words)
