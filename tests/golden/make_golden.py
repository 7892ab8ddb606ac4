"""Generates the golden fixtures in this folder from the reference itself.

The reference's tick, compiled for the host from its own sources
(oracle/_ref/libcarlref_cpu.so, `make -C oracle cpu arena`), is run on small
seeded cases and its outputs are stored:

  arena.json            sizes and SHA-256 of every arena table
                        (src/ArenaMesh.cu:15-125)
  kickoff_4v4.npz       the kickoff permutation table (src/RLConstants.cu:4-29)
                        and car positions after reset() for 96 sims
                        (include/State/Reset.cuh:52-171)
  tick_<case>.npz       a warmed-up state, direct controls, the state after 1
                        and after 8 ticks, and the tick-1 broadphase cells,
                        candidate counts and SAT pair sets (src/Kernels.cu:15-202)
  env_step_1v1.npz      obs/state/rewards/dones of 4 RL steps with discrete
                        actions and frameskip 2 (src/EnvIO.cu:47-135,565-643)

Run from the repository root:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from carl_b200 import capi, workloads  # noqa: E402
from oracle.refenv import RefCpu, reference_arena_tables, reference_kickoff_table  # noqa: E402

TICK_CASES = {
    # name: (n_sim, n_blue, n_orange, scenario, seed)
    "2v2_mixed": (12, 2, 2, "mixed", 21),
    "3v3_crowd": (8, 3, 3, "crowd", 22),
    "1v1_floor": (16, 1, 1, "floor", 23),
}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_arena() -> None:
    ref = RefCpu(1, 1, 1, 0)
    t = reference_arena_tables(ref)
    ref.close()
    doc = {k: {"shape": list(v.shape), "dtype": str(v.dtype), "sha256": sha(v)} for k, v in t.items()}
    (HERE / "arena.json").write_text(json.dumps(doc, indent=1) + "\n")


def make_kickoff() -> None:
    ref = RefCpu(96, 4, 4, 7)
    ref.reset()
    np.savez_compressed(HERE / "kickoff_4v4.npz", seed=7, table=reference_kickoff_table(),
                        car_pos=ref.read_field("CAR_POS"), car_rot=ref.read_field("CAR_ROT"))
    ref.close()


def make_tick(name: str) -> None:
    n_sim, nb, no, scenario, seed = TICK_CASES[name]
    ref = RefCpu(n_sim, nb, no, seed)
    getattr(workloads, scenario + "_state")(ref, seed)
    rng = np.random.default_rng(seed + 1)
    ref.ticks(2, workloads.controls(rng, n_sim * (nb + no)), 8)
    s0 = ref.snapshot()
    ctl = workloads.controls(rng, n_sim * (nb + no))
    ref.ticks(2, ctl, 1)
    s1 = ref.snapshot()
    diag = {f: ref.read_field(f) for f in ("DIAG_CELL_IDX", "DIAG_NUM_TRIS", "DIAG_SAT_PAIRS")}
    ref.ticks(2, ctl, 7)
    s8 = ref.snapshot()
    ref.close()
    arrays = {"dims": np.array([n_sim, nb, no, seed], np.int32), "controls": ctl}
    for tag, snap in (("s0", s0), ("s1", s1), ("s8", s8)):
        for field, words in snap.items():
            arrays[f"{tag}/{field}"] = words
    for field, words in diag.items():
        arrays[f"d1/{field}"] = words
    np.savez_compressed(HERE / f"tick_{name}.npz", **arrays)


def make_env_step() -> None:
    n_sim, nb, no, seed = 8, 1, 1, 31
    ref = RefCpu(n_sim, nb, no, seed, frameskip=2)
    ref.reset()
    rng = np.random.default_rng(seed)
    arrays = {"dims": np.array([n_sim, nb, no, seed, 2], np.int32)}
    bufs = {"obs": capi.BUF_OBS, "state": capi.BUF_STATE, "rewards": capi.BUF_REWARDS, "dones": capi.BUF_DONES,
            "episode_ticks": capi.BUF_EPISODE_TICKS, "transition_obs": capi.BUF_TRANSITION_OBS}
    for step in range(4):
        a = workloads.discrete_actions(rng, n_sim * (nb + no))
        ref.env_step(0, a)
        arrays[f"actions/{step}"] = a
        for k, b in bufs.items():
            arrays[f"{k}/{step}"] = ref.get_buffer(b)
    ref.close()
    np.savez_compressed(HERE / "env_step_1v1.npz", **arrays)


if __name__ == "__main__":
    make_arena()
    make_kickoff()
    for case in TICK_CASES:
        make_tick(case)
    make_env_step()
    for p in sorted(HERE.glob("*")):
        print(f"{p.name:24s} {p.stat().st_size:8d} B")
