"""Writes tests/golden/front_end_*.npz: output buffers of this project's drop-in
front end (carl_b200.carl.Env, the `_carl` replacement) after a few env steps,
with the snapshot words they were packed from and the device action mask.

tests/test_reference_python_layer.py runs the reference's own Python layer
(python/carl/gymnasium/state.py and action.py, imported from its source tree
with carl_b200.carl installed as `carl._carl`) over these buffers: the state
views, the action codec, and the reward context of the last step (the previous
step's state and obs are saved with their snapshot words for that).  The
reference's Python sources cannot be run on the GPU machine and its CUDA module
cannot be run on the CPU machine, so the buffers cross as fixtures.

Run on a machine with a CUDA device:  python tests/golden/make_front_end_fixture.py [out_dir]
TEST INFRASTRUCTURE.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

CASES = {
    # name: (n_sim, n_blue, n_orange, seed, frameskip, invert_orange, normalize, previous_controls)
    "front_end_2v2": (16, 2, 2, 41, 8, True, False, False),
    "front_end_1v2_options": (12, 1, 2, 43, 2, False, True, True),
}
SNAPSHOT_FIELDS = ["CAR_POS", "CAR_VEL", "CAR_ANG", "CAR_ROT", "CAR_IS_DEMOED", "CAR_INTERNAL", "BALL_POS",
                   "BALL_VEL", "BALL_ANG", "PAD_COOLDOWNS", "GOALS", "EPISODE_TICKS", "CAR_WHEEL_CONTACT"]


def make(name, n_sim, nb, no, seed, frameskip, invert, normalize, prev) -> dict:
    import torch

    from carl_b200 import carl as front
    from carl_b200 import workloads
    from carl_b200.action import CARLActionCodec

    env = front.Env(n_sim, nb, no, seed, frameskip, invert, normalize, prev)
    workloads.mixed_state(env._env, seed + 1)
    rng = np.random.default_rng(seed + 2)
    out = {"dims": np.array([n_sim, nb, no, seed, frameskip, int(invert), int(normalize), int(prev)])}
    for step in range(3):
        if step == 2:
            # The previous step's state, obs and snapshot words (the reward context's
            # `previous` side).
            torch.cuda.synchronize()
            out["prev_state"] = env.get_state().cpu().numpy()
            out["prev_obs"] = obs.cpu().numpy()
            env._env.synchronize()
            for f in SNAPSHOT_FIELDS:
                out[f"prev_snap/{f}"] = env._env.read_field(f)
        actions = workloads.discrete_actions(rng, n_sim * (nb + no)).reshape(n_sim, nb + no, 7)
        obs = env.step(torch.from_numpy(actions).cuda())
        torch.cuda.current_stream().wait_stream(torch.cuda.ExternalStream(env.stream))
        out[f"actions/{step}"] = actions
    torch.cuda.synchronize()
    out["transition_score_difference"] = env.get_transition_score_difference().cpu().numpy()
    out["transition_episode_ticks"] = env.get_transition_episode_ticks().cpu().numpy()
    out["transition_overtime"] = env.get_transition_overtime().cpu().numpy()
    out["obs"] = obs.cpu().numpy()
    out["state"] = env.get_state().cpu().numpy()
    out["transition_obs"] = env.get_transition_obs().cpu().numpy()
    out["transition_state"] = env.get_transition_state().cpu().numpy()
    out["rewards"] = env.get_rewards().cpu().numpy()
    out["dones"] = env.get_dones().cpu().numpy()
    out["mask"] = CARLActionCodec(previous_controls=prev).mask(obs).cpu().numpy()
    env._env.synchronize()
    for f in SNAPSHOT_FIELDS:
        out[f"snap/{f}"] = env._env.read_field(f)
    env.close()
    return out


def main() -> None:
    out_dir = Path(sys.argv[1]) if len(sys.argv) > 1 else HERE
    for name, args in CASES.items():
        np.savez_compressed(out_dir / f"{name}.npz", **make(name, *args))
        print("wrote", out_dir / f"{name}.npz")


if __name__ == "__main__":
    main()
