"""Drop-in front end of the reference's native module (``carl._carl``).

Same class and method names, argument meanings and error behaviour as the
reference's pybind11 module (jwmccarthy/CARL python/carl.cu:286-988):

* ``Env(n_sim, n_blue, n_orange, seed, frameskip=1, invert_orange=True,
  normalize=False, previous_controls=False)``, plus the B200 additions
  ``device`` (CUDA ordinal, default: torch's current device) and ``sim_offset``
  (global index of this env's first sim, for sharding over GPUs);
* ``step`` / ``step_continuous`` take ``[n_sim, n_cars, 7]`` int32 / float32 CUDA
  tensors and return the observation buffer;
* ``get_*`` return views of the env's output buffers, overwritten in place by
  the next call (the reference returns non-owning DLPack capsules of the same
  buffers; ``torch.from_dlpack`` accepts either);
* dtype errors raise ``TypeError``; device, shape, stride and range errors raise
  ``ValueError``; CUDA failures raise ``RuntimeError``.  All validation happens
  before any state changes.

Device inputs are ordered onto the env's stream after torch's current stream,
and stay referenced until the env has read them (the reference's
``__dlpack__(stream=env_stream)`` handoff).
"""

from __future__ import annotations

import torch

from . import capi

# ---- module constants (python/carl.cu:825-909) ------------------------------
ACTION_NVECS = (3, 3, 3, 2, 2, 3, 2)
ACTION_LOGITS = sum(ACTION_NVECS)
CONTINUOUS_ACTION_LOW = (-1.0, -1.0, -1.0, 0.0, 0.0, -1.0, 0.0)
CONTINUOUS_ACTION_HIGH = (1.0,) * 7
_LOGIT_OFFSETS = [sum(ACTION_NVECS[:i]) for i in range(len(ACTION_NVECS))]
# Action fields: horizontal, vertical, throttle, powerslide, boost, air roll, jump.
ACTION_PITCH_LOGITS = slice(_LOGIT_OFFSETS[1] + 1, _LOGIT_OFFSETS[1] + ACTION_NVECS[1], None)
ACTION_AIR_ROLL_LOGITS = slice(_LOGIT_OFFSETS[5] + 1, _LOGIT_OFFSETS[5] + ACTION_NVECS[5], None)
ACTION_POWERSLIDE_LOGIT = _LOGIT_OFFSETS[3] + 1
ACTION_BOOST_LOGIT = _LOGIT_OFFSETS[4] + 1
ACTION_JUMP_LOGIT = _LOGIT_OFFSETS[6] + 1

OBS_VECTOR_SIZE = 3
OBS_POS = 0
OBS_VEL = 3
OBS_ANG = 6
OBS_FORWARD = 9
OBS_UP = 12
OBS_BOOST = 15
OBS_ON_GROUND = 16
OBS_DEMOED = 17
OBS_HAS_FLIPPED = 18
OBS_HAS_DOUBLE_JUMPED = 19
OBS_IS_BOOSTING = 20
STATE_BALL_TOUCH = 21
OBS_BALL = OBS_FORWARD
OBS_PER_CAR = STATE_BALL_TOUCH
STATE_PER_CAR = STATE_BALL_TOUCH + 1
NUM_BOOST_PADS = 34
OBS_BOOST_PADS = 2 * NUM_BOOST_PADS
OBS_RELATIVE_EGO_BALL = 2 * OBS_VECTOR_SIZE
OBS_RELATIVE_PER_OTHER_CAR = OBS_RELATIVE_EGO_BALL
OBS_RELATIVE_GOALS = 2 * OBS_VECTOR_SIZE
OBS_EGO_DODGE = 2
OBS_EGO_BOOST_INDEX = OBS_BALL + OBS_BOOST
OBS_EGO_ON_GROUND_INDEX = OBS_BALL + OBS_ON_GROUND
OBS_EGO_CONTROLLER = 5
OBS_PREVIOUS_CONTROLS = 8
OBS_CONTROLLER_VERSION = 3
OBS_EGO_FLIP_INDEX = -OBS_EGO_DODGE - OBS_EGO_CONTROLLER
OBS_EGO_DODGE_TIME_INDEX = OBS_EGO_FLIP_INDEX + 1
CAR_INTERNAL_SIZE = 19

PHYS_TICKS_PER_SECOND = 120
PHYS_DT = 1.0 / PHYS_TICKS_PER_SECOND
DOUBLEJUMP_MAX_DELAY = 1.25
REGULATION_TICKS = 5 * 60 * PHYS_TICKS_PER_SECOND
OBS_POSITION_SCALE = (4108.0, 6000.0, 2076.0)
BALL_MAX_SPEED = 6000.0
BALL_MAX_ANG_SPEED = 6.0
CAR_MAX_SPEED = 2300.0
CAR_MAX_ANG_SPEED = 5.5
BOOST_MAX = 100.0
BOOST_PAD_POSITIONS = (
    (-3584.0, 0.0, 73.0), (3584.0, 0.0, 73.0), (-3072.0, 4096.0, 73.0), (3072.0, 4096.0, 73.0),
    (-3072.0, -4096.0, 73.0), (3072.0, -4096.0, 73.0), (0.0, -4240.0, 70.0), (-1792.0, -4184.0, 70.0),
    (1792.0, -4184.0, 70.0), (-940.0, -3308.0, 70.0), (940.0, -3308.0, 70.0), (0.0, -2816.0, 70.0),
    (-3584.0, -2484.0, 70.0), (3584.0, -2484.0, 70.0), (-1788.0, -2300.0, 70.0), (1788.0, -2300.0, 70.0),
    (-2048.0, -1036.0, 70.0), (0.0, -1024.0, 70.0), (2048.0, -1036.0, 70.0), (-1024.0, 0.0, 70.0),
    (1024.0, 0.0, 70.0), (-2048.0, 1036.0, 70.0), (0.0, 1024.0, 70.0), (2048.0, 1036.0, 70.0),
    (-1788.0, 2300.0, 70.0), (1788.0, 2300.0, 70.0), (-3584.0, 2484.0, 70.0), (3584.0, 2484.0, 70.0),
    (0.0, 2816.0, 70.0), (-940.0, 3308.0, 70.0), (940.0, 3308.0, 70.0), (-1792.0, 4184.0, 70.0),
    (1792.0, 4184.0, 70.0), (0.0, 4240.0, 70.0),
)

_TORCH_DTYPE = {capi.DT_F32: torch.float32, capi.DT_I32: torch.int32, capi.DT_BOOL: torch.bool,
                capi.DT_I64: torch.int64}
_TYPESTR = {torch.float32: "<f4", torch.int32: "<i4", torch.bool: "|b1", torch.int64: "<i8", torch.uint8: "|u1"}


class _DeviceBuffer:
    """CUDA Array Interface view of an env-owned buffer (keeps the env alive)."""

    def __init__(self, owner, ptr: int, shape: tuple, dtype: torch.dtype):
        self._owner = owner
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": _TYPESTR[dtype], "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def _as_tensor(x) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x
    if hasattr(x, "__dlpack__"):
        return torch.from_dlpack(x)
    raise TypeError(f"expected a tensor, got {type(x).__name__}")


class Env:
    """A batch of independent 1v1 .. 4v4 Rocket League arenas on one GPU."""

    def __init__(self, n_sim: int, n_blue: int, n_orange: int, seed: int, frameskip: int = 1,
                 invert_orange: bool = True, normalize: bool = False, previous_controls: bool = False,
                 *, device: int | None = None, sim_offset: int = 0):
        if frameskip < 1:
            raise ValueError("frameskip must be at least 1")
        if device is None:
            device = torch.cuda.current_device()
        try:
            self._env = capi.Env(n_sim, n_blue, n_orange, seed, frameskip=frameskip, invert_orange=invert_orange,
                                 normalize=normalize, previous_controls=previous_controls, device=device,
                                 sim_offset=sim_offset)
        except capi.CarlbError as exc:
            raise (ValueError if exc.status == capi.ERR_VALUE else RuntimeError)(str(exc)) from None
        self._device = torch.device("cuda", device)
        self._frameskip = frameskip
        self._views: dict[int, torch.Tensor] = {}

    # ---- validation (python/carl.cu:101-278) ----
    def _device_ok(self, t: torch.Tensor, name: str) -> None:
        if t.device != self._device:
            raise ValueError(f"{name} must be on {self._device}")

    def _check(self, x, name: str, shape: tuple, dtypes, *, type_msg: str | None = None) -> torch.Tensor:
        t = _as_tensor(x)
        if t.dtype not in dtypes:
            raise TypeError(type_msg or f"{name} has an invalid dtype")
        self._device_ok(t, name)
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name} has an invalid shape")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        return t

    def _actions(self, actions, dtype: torch.dtype, what: str) -> torch.Tensor:
        t = _as_tensor(actions)
        if t.dtype != dtype:
            raise TypeError(f"{what} must have dtype {str(dtype).replace('torch.', '')}")
        self._device_ok(t, what)
        if tuple(t.shape) != (self.n_sim, self.n_cars, 7):
            raise ValueError(f"{what} must have shape [n_sim, n_cars, 7]")
        if not t.is_contiguous():
            raise ValueError(f"{what} must be contiguous")
        return t

    def _selection(self, indices) -> tuple[torch.Tensor | None, int]:
        if indices is None:
            return None, self.n_sim
        t = _as_tensor(indices)
        if t.dtype != torch.int64:
            raise TypeError("simulation_indices must have dtype int64")
        self._device_ok(t, "simulation_indices")
        if t.dim() != 1:
            raise ValueError("simulation_indices must be one-dimensional")
        if not t.is_contiguous():
            raise ValueError("simulation_indices must be contiguous")
        if t.shape[0] > self.n_sim:
            raise ValueError("too many simulation_indices")
        return t, int(t.shape[0])

    def _call(self, fn, *args):
        try:
            fn(*args)
        except capi.CarlbError as exc:
            kind = {capi.ERR_VALUE: ValueError, capi.ERR_TYPE: TypeError}.get(exc.status, RuntimeError)
            raise kind(str(exc)) from None

    # ---- stepping ----
    def step(self, actions) -> torch.Tensor:
        """One RL step with discrete actions; returns the observation buffer."""
        t = self._actions(actions, torch.int32, "actions")
        self._call(self._env.env_step, capi.ACTIONS_DISCRETE, t)
        return self.get_obs()

    def step_continuous(self, actions) -> torch.Tensor:
        """One RL step with continuous actions; returns the observation buffer."""
        t = self._actions(actions, torch.float32, "continuous actions")
        self._call(self._env.env_step, capi.ACTIONS_CONTINUOUS, t)
        return self.get_obs()

    def reset(self) -> None:
        self._call(self._env.reset)

    # ---- state injection (python/carl.cu:384-706) ----
    def apply_reset_state(self, ball_position, ball_velocity, ball_angular_velocity, car_position, car_rotation,
                          car_velocity, car_angular_velocity, car_demoed, car_boost=None, car_internal_state=None,
                          blue_score=None, orange_score=None, episode_ticks=None, simulation_indices=None,
                          reset_mask=None) -> None:
        if reset_mask is not None and simulation_indices is not None:
            raise ValueError("specify reset_mask or simulation_indices, not both")
        idx, k = self._selection(simulation_indices)
        mask = None
        if reset_mask is not None:
            mask = self._check(reset_mask, "reset_mask", (self.n_sim,), (torch.bool,))
            k = self.n_sim
        nc = self.n_cars
        f32 = (torch.float32,)
        bp = self._check(ball_position, "ball_position", (k, 3), f32)
        bv = self._check(ball_velocity, "ball_velocity", (k, 3), f32)
        ba = self._check(ball_angular_velocity, "ball_angular_velocity", (k, 3), f32)
        cp = self._check(car_position, "car_position", (k, nc, 3), f32)
        cr = self._check(car_rotation, "car_rotation", (k, nc, 4), f32)
        cv = self._check(car_velocity, "car_velocity", (k, nc, 3), f32)
        ca = self._check(car_angular_velocity, "car_angular_velocity", (k, nc, 3), f32)
        cd = self._check(car_demoed, "car_demoed", (k, nc), (torch.bool, torch.int32))
        boost = None if car_boost is None else self._check(car_boost, "car_boost", (k, nc), f32)
        internal = None if car_internal_state is None else self._check(
            car_internal_state, "car_internal_state", (k, nc, CAR_INTERNAL_SIZE), f32)
        match = [blue_score, orange_score, episode_ticks]
        if any(m is not None for m in match) and not all(m is not None for m in match):
            raise ValueError("blue_score, orange_score and episode_ticks must be supplied together")
        blue = orange = ticks = None
        if blue_score is not None:
            blue = self._check(blue_score, "blue_score", (k,), (torch.int32,))
            orange = self._check(orange_score, "orange_score", (k,), (torch.int32,))
            ticks = self._check(episode_ticks, "episode_ticks", (k,), (torch.int32,))
        if k == 0:
            return
        self._call(self._env.apply_reset_state, k, bp, bv, ba, cp, cr, cv, ca, cd, cd.dtype == torch.bool, boost,
                   internal, blue, orange, ticks, idx, mask)
        if mask is None:
            self._env.synchronize()

    def set_ball(self, position, velocity, angular_velocity, simulation_indices=None) -> None:
        idx, k = self._selection(simulation_indices)
        f32 = (torch.float32,)
        p = self._check(position, "position", (k, 3), f32)
        v = self._check(velocity, "velocity", (k, 3), f32)
        a = self._check(angular_velocity, "angular_velocity", (k, 3), f32)
        self._call(self._env.set_ball, k, p, v, a, idx)

    def set_car(self, position, rotation, velocity, angular_velocity, demoed, boost=None, internal_state=None,
                simulation_indices=None) -> None:
        idx, k = self._selection(simulation_indices)
        nc = self.n_cars
        f32 = (torch.float32,)
        p = self._check(position, "position", (k, nc, 3), f32)
        r = self._check(rotation, "rotation", (k, nc, 4), f32)
        v = self._check(velocity, "velocity", (k, nc, 3), f32)
        a = self._check(angular_velocity, "angular_velocity", (k, nc, 3), f32)
        d = self._check(demoed, "demoed", (k, nc), (torch.bool, torch.int32))
        b = None if boost is None else self._check(boost, "boost", (k, nc), f32)
        s = None if internal_state is None else self._check(internal_state, "internal_state",
                                                            (k, nc, CAR_INTERNAL_SIZE), f32)
        self._call(self._env.set_car, k, p, r, v, a, d, d.dtype == torch.bool, b, s, idx)

    def set_match_state(self, blue_score, orange_score, episode_ticks, simulation_indices=None) -> None:
        idx, k = self._selection(simulation_indices)
        i32 = (torch.int32,)
        b = self._check(blue_score, "blue_score", (k,), i32)
        o = self._check(orange_score, "orange_score", (k,), i32)
        t = self._check(episode_ticks, "episode_ticks", (k,), i32)
        self._call(self._env.set_match_state, k, b, o, t, idx)

    def reset_boost_pads(self, simulation_indices=None) -> None:
        idx, k = self._selection(simulation_indices)
        self._call(self._env.reset_boost_pads, k, idx)
        self._env.synchronize()

    # ---- outputs (non-owning views, overwritten in place) ----
    def _buffer(self, which: int) -> torch.Tensor:
        view = self._views.get(which)
        if view is None:
            ptr, shape, dt = self._env.buffer(which)
            dtype = _TORCH_DTYPE[dt]
            view = torch.as_tensor(_DeviceBuffer(self, ptr, shape, dtype), device=self._device)
            self._views[which] = view
        return view

    def get_obs(self):
        return self._buffer(capi.BUF_OBS)

    def get_transition_obs(self):
        return self._buffer(capi.BUF_TRANSITION_OBS)

    def get_state(self):
        return self._buffer(capi.BUF_STATE)

    def get_transition_state(self):
        return self._buffer(capi.BUF_TRANSITION_STATE)

    def get_rewards(self):
        return self._buffer(capi.BUF_REWARDS)

    def get_dones(self):
        return self._buffer(capi.BUF_DONES)

    def get_score_difference(self):
        return self._buffer(capi.BUF_SCORE_DIFFERENCE)

    def get_episode_ticks(self):
        return self._buffer(capi.BUF_EPISODE_TICKS)

    def get_transition_score_difference(self):
        return self._buffer(capi.BUF_TRANSITION_SCORE_DIFFERENCE)

    def get_transition_episode_ticks(self):
        return self._buffer(capi.BUF_TRANSITION_EPISODE_TICKS)

    def get_overtime(self):
        return self._buffer(capi.BUF_OVERTIME)

    def get_transition_overtime(self):
        return self._buffer(capi.BUF_TRANSITION_OVERTIME)

    # ---- properties ----
    def _set_limit(self, which: int, value: int) -> None:
        self._call(self._env.set_limit, which, int(value))

    max_ticks = property(None, lambda self, v: self._set_limit(capi.LIMIT_MAX_TICKS, v))
    overtime_timeout_ticks = property(None, lambda self, v: self._set_limit(capi.LIMIT_OVERTIME_TIMEOUT_TICKS, v))
    no_touch_timeout_ticks = property(None, lambda self, v: self._set_limit(capi.LIMIT_NO_TOUCH_TIMEOUT_TICKS, v))

    @property
    def frameskip(self) -> int:
        return self._env.get_limit(capi.LIMIT_FRAMESKIP)

    @frameskip.setter
    def frameskip(self, value: int) -> None:
        self._set_limit(capi.LIMIT_FRAMESKIP, value)

    @property
    def obs_dim(self) -> int:
        return self._env.obs_dim

    @property
    def act_dim(self) -> int:
        return self._env.act_dim

    @property
    def action_nvec(self) -> tuple:
        return ACTION_NVECS

    @property
    def n_sim(self) -> int:
        return self._env.n_sim

    @property
    def n_cars(self) -> int:
        return self._env.n_cars

    @property
    def stream(self) -> int:
        """The env's cudaStream_t as an integer (for torch.cuda.ExternalStream)."""
        return self._env.stream

    def close(self) -> None:
        self._views.clear()
        self._env.close()
