"""Throughput benchmark of the batched Rocket League tick on B200.

Default workload (config C3): 3v3, n_sim = 32768 sims per GPU, default arena,
seeded synthetic initial states (cars uniform over the field floor, planar
velocity N(0, 800 uu/s), yaw uniform, boost U[0, 100], ball at rest at centre)
and direct controls redrawn every 8 ticks (throttle/steer/pitch/yaw/roll
U[-1, 1], jump/boost/handbrake Bernoulli(0.3)).  The tick runs in the default
mode (compat_flags = 0), which reproduces the reference's CUDA build and is the
mode the parity tests hold to the strict gates.

A *step* is one control period: the controls for all cars are staged on the
device and 8 physics ticks run (one replay of the captured stage-kernel graph).
The metric is agent-steps/s = cars x ticks / s, one agent-step being one car
advanced one 120 Hz tick.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                  [--workload c3|c1|c4|c5|step|mask]

  c1    1v1, n_sim = 1024 per GPU, kickoff resets (the launch-overhead regime)
  c4    2v2, 262,144 sims over 8 GPUs (32,768 per GPU), 50 % airborne, 25 % on
        walls / ceiling, 25 % near corners and goal mouths
  c5    4v4, 1,048,576 sims over 8 GPUs (131,072 per GPU), the C4 states, env
        steps at frameskip 1 with 1 % of sims reset to kickoff by a masked
        apply_reset_state each step and the obs handed to torch each step
  step  env steps (ticks + packing) at frameskip 8 (C2 with --blue 1 --orange 1
        --n-sim 65536 --frameskip 1)
  mask  device action masks of a C5 shard's observations

For N > 1 it runs under torch.distributed.run, one rank per GPU; each rank
simulates its own contiguous slice of sims (global sim offset rank*n_sim), so
per-GPU work is fixed (weak scaling) and there is no collective in the tick.

Timed region: barrier + synchronize, K steps enqueued back to back (no host
synchronisation between them), synchronize + barrier.  Each step's device time
is taken with CUDA events on the env stream; before each timed step a 256 MiB
buffer is written on the same stream (outside the events) to flush the 126 MB
L2.  The value uses the maximum over ranks of the summed step times.  Stage
kernel times, work-list sizes and the per-stage rooflines come from a separate
pass after the timed region (events around each stage kernel of the first sim
slice, last tick of each step).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

TICKS_PER_STEP = 8
FLUSH_BYTES = 256 << 20
# Byte model CARLB-v1 of a whole tick: persistent tick state read once and
# written once per tick, packed fp32 (vec3 12 B, quat 16 B, ints 4 B), plus the
# actions read.
BYTES_PER_CAR_TICK = 620
BYTES_PER_SIM_TICK = 504
# Algorithmic bytes of each stage kernel: the words the stage must read and
# write per car and per sim of its slice, and per entry of the work lists it
# runs over (arena tables are L2-resident and excluded).
#   flat      pose in (pos, vel, ang, cen, rot: 16 words), candidate list start,
#             count, SAT hit mask (9 words) and ray keys (8 words) out, episode
#             tick read-modify-write per sim.
#   ray       own pose (centre, rotation: 7 words), demolition flag, ray keys (8
#             words) and candidate start in, rays (16 words) and wheel bits out;
#             ball position per sim.
#   ctlSusp   controls and suspension: actions (8), control state (24), staging
#             (15), velocities, rays, body, friction and manifold state, SAT hit
#             words in (about 102 words); control state, staging, friction and
#             velocities or the contact hand-over out (about 60 words).
#   contact   per listed car: hand-over velocities (18 words), pose, candidate
#             range and hit mask in (20 words), pose, velocities and manifold
#             count and normal out (20 words).
#   carCar    the pair gate of every sim: box centre and demolition flag of
#             each car (4 words); per sim with a pair in reach: every car's
#             pose, velocities, impulse and contact state in and out (2 x 24
#             words per car).
#   ball      per moving ball: ball state and hand-over values in (27 words),
#             velocities and push velocity out (9 words).
#   finish    per car: pose, velocities, impulse, demolition and respawn state,
#             boost and controls in (34 words), pose, velocities, impulse and
#             finish state out (22 words); per sim: ball state and hand-over
#             values in (40 words) and out (26 words), 34 pad cooldowns and the
#             goal state in and out (78 words).
#   ballPrep  ball state in (22 words), hand-over values out (15 words).
STAGE_BYTES = {
    # stage: (bytes per car, bytes per sim, {work list: bytes per entry})
    "ballPrep": (0, 148, {}),
    "flat": (140, 8, {}),
    "ray": (136, 12, {}),
    "ctlSusp": (648, 0, {}),
    "contact": (0, 0, {"plane_cars": 232, "sat_cars": 232}),
    "carCar": (16, 0, {"car_car_sims_cars": 192}),
    "ball": (0, 0, {"moving_balls": 144}),
    "finish": (224, 576, {}),
}
UNIT = "agent-steps/s"


def metric_name(args) -> str:
    if args.workload == "c1":
        return "agent-steps/sec at 1v1 n_sim=1024 (C1)"
    if args.workload == "c4":
        return "agent-steps/sec at 2v2 n_sim=32768 per GPU (C4)"
    return f"agent-steps/sec at {args.blue}v{args.orange} n_sim={args.n_sim}"


def bytes_per_agent_tick(n_cars: int) -> float:
    return (n_cars * BYTES_PER_CAR_TICK + BYTES_PER_SIM_TICK) / n_cars


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--n-sim", type=int, default=32768, help="sims per GPU")
    ap.add_argument("--blue", type=int, default=3)
    ap.add_argument("--orange", type=int, default=3)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-stages", action="store_true", help="skip the stage-timing pass")
    ap.add_argument("--workload", choices=["c3", "c1", "c4", "c5", "reset", "step", "mask"], default="c3",
                    help="c3: the headline tick throughput; c1 / c4: the other tick configs; c5 (alias reset): env "
                         "steps with masked resets and obs handed to torch; step: env steps at frameskip 8; "
                         "mask: device action masks")
    ap.add_argument("--reset-n-sim", type=int, default=131072, help="sims per GPU of the c5 workload (4v4)")
    ap.add_argument("--frameskip", type=int, default=TICKS_PER_STEP,
                    help="ticks per env step of the step workload (1 with --blue 1 --orange 1 --n-sim 65536: "
                         "config C2, obs packed every tick)")
    args = ap.parse_args()
    if args.workload == "reset":
        args.workload = "c5"
    if args.workload == "c1":
        args.blue, args.orange, args.n_sim = 1, 1, 1024
    elif args.workload == "c4":
        args.blue, args.orange, args.n_sim = 2, 2, 32768
    return args


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed
    region, for the GPUs of this run (one sampler per node, on local rank 0)."""

    QUERY = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, devices: list[int]):
        self.bus_ids = set()
        try:
            import torch

            for d in devices:
                pr = torch.cuda.get_device_properties(d)
                self.bus_ids.add(f"{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0")
        except Exception:
            pass
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.25)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = []
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            # nvidia-smi prints domain:bus:device.function; compare bus:device.function.
            if self.bus_ids and f[1].lower()[-7:] not in self.bus_ids:
                continue
            rows.append(f)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        reasons = sorted({name for r in rows for name, v in zip(self.REASONS, r[6:10]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "gpus": len(self.bus_ids)}


# ------------------------------------------------------------ workload ----
def initial_state(args, env, seed: int) -> None:
    """The workload's seeded initial state (C3 floor, C1 kickoff, C4 mixed)."""
    from carl_b200 import workloads

    if args.workload == "c1":
        env.reset()
    elif args.workload == "c4":
        workloads.mixed_state(env, seed)
    else:
        workloads.floor_state(env, seed)


def workload_name(args) -> str:
    if args.workload == "c1":
        return "C1 1v1 n_sim=1024 per GPU, kickoff reset, direct controls held 8 ticks"
    if args.workload == "c4":
        return ("C4 2v2 n_sim=32768 per GPU (262,144 over 8 GPUs), 50% airborne / 25% walls and ceiling / "
                "25% corners and goal mouths, direct controls held 8 ticks")
    return f"C3 {args.blue}v{args.orange} n_sim={args.n_sim} per GPU, direct controls held 8 ticks"


def data_name(args) -> str:
    states = {"c1": "kickoff states", "c4": "C4 mixed states"}.get(args.workload, "C3 floor states")
    return f"synthetic (seeded {states}, direct controls redrawn every 8 ticks)"


def make_env(args, rank: int, device: int):
    from carl_b200 import capi

    env = capi.Env(args.n_sim, args.blue, args.orange, seed=args.seed, device=device,
                   sim_offset=rank * args.n_sim)
    initial_state(args, env, args.seed + 1000 * rank)
    return env


def control_pool(n_cars_total: int, count: int, seed: int):
    from carl_b200 import workloads

    rng = np.random.default_rng(seed)
    return [workloads.controls(rng, n_cars_total) for _ in range(count)]


def traffic_per_launch(stage: str, n_sim: int) -> float | None:
    """DRAM bytes per launch of a stage kernel, from the committed ncu summaries
    (stated for a slice of the n_sim = 32768 bench; traffic grows with the sims,
    so it is scaled to this run's n_sim).  None when not captured."""
    key = f"traffic_bytes_per_launch[{stage}]:"
    for path in sorted((ROOT / "profiles").glob("*.md")):
        for line in path.read_text().splitlines():
            if line.startswith(key):
                return float(line.split(":", 1)[1].split()[0]) * n_sim / 32768
    return None


def world_groups(args) -> int:
    """Sim slices the library steps concurrently (CARLB_GROUPS, default 2; one
    slice per 4096 sims at most)."""
    g = int(os.environ.get("CARLB_GROUPS", "2"))
    return max(1, min(8, g, args.n_sim // 4096))


def launches_per_step(groups: int) -> int:
    """Kernels of the library launched per step: 8 stage kernels per tick and slice,
    plus, with graph replay (the default), the kernel that sets the tick counter."""
    graph = os.environ.get("CARLB_GRAPH", "1") != "0"
    return 8 * TICKS_PER_STEP * groups + (1 if graph else 0)


def fp32_flops_per_car_tick() -> float | None:
    """FP32 FLOPs per car per tick summed over the stage kernels, from the
    committed ncu summary (sass thread fadd/fmul/ffma counts)."""
    import re

    try:
        text = (ROOT / "profiles" / "staged_tick_3v3_32768.md").read_text()
    except OSError:
        return None
    vals = [float(m.group(1)) for m in re.finditer(r"fp32_flops_per_car_tick\[\w+\]: (\d+(?:\.\d+)?)", text)]
    return sum(vals) if vals else None


def measured_hbm_peak() -> tuple[float, str]:
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def stage_bytes(stage: str, cars: float, sims: float, work: dict) -> float:
    """Algorithmic bytes of one launch of `stage` over `cars` cars and `sims`
    sims, with the work-list sizes `work` of the same slice."""
    per_car, per_sim, per_entry = STAGE_BYTES[stage]
    total = per_car * cars + per_sim * sims
    for name, b in per_entry.items():
        if name == "car_car_sims_cars":
            total += b * work.get("car_car_sims", 0) * (cars / max(sims, 1))
        else:
            total += b * work.get(name, 0)
    return total


# -------------------------------------------------------- reference CPU ----
def reference_cpu_time(snapshot, n_sim, n_blue, n_orange, seed, controls, steps, threads):
    """Times the reference's tick compiled for the host (OpenMP over sims).

    Returns (agent-steps/s, seconds, threads used)."""
    from oracle.refenv import RefCpu

    used = RefCpu.set_threads(threads)
    ref = RefCpu(n_sim, n_blue, n_orange, seed)
    ref.restore(snapshot)
    ref.ticks(2, controls[0], 1)  # touch pages / spin up the thread pool
    t0 = time.perf_counter()
    for i in range(steps):
        ref.ticks(2, controls[i % len(controls)], TICKS_PER_STEP)
    dt = time.perf_counter() - t0
    ref.close()
    return n_sim * (n_blue + n_orange) * TICKS_PER_STEP * steps / dt, dt, used


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------- arms --------
def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the reference's own CPU tick on the host cores, plus
    its CUDA build on the same states and controls when a GPU is present."""
    if rank != 0:
        return
    from oracle.refenv import RefCpu

    n_cars = args.blue + args.orange
    # The initial state is built on the host build of the reference so the arm
    # needs no GPU for its headline value.
    threads = host_threads()
    RefCpu.set_threads(threads)
    ref = RefCpu(args.n_sim, args.blue, args.orange, args.seed)
    initial_state(args, ref, args.seed)
    snap = ref.snapshot()
    ref.close()
    pool_n = max(4, min(16, args.steps + args.warmup))
    ctl = control_pool(args.n_sim * n_cars, pool_n, args.seed + 1)
    steps = max(1, min(args.steps, 8 if args.n_sim * n_cars > 50000 else 200))
    warm = max(0, min(args.warmup, 1))
    if warm:
        reference_cpu_time(snap, args.n_sim, args.blue, args.orange, args.seed, ctl, warm, threads)
    value, secs, used = reference_cpu_time(snap, args.n_sim, args.blue, args.orange, args.seed, ctl, steps, threads)
    sample = (f"{steps} steps x {TICKS_PER_STEP} ticks of the full {args.blue}v{args.orange} n_sim={args.n_sim} "
              f"workload ({secs:.1f} s), OpenMP over sims")
    line = {
        "impl": "reference", "metric": metric_name(args), "value": value, "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": secs * 1e3 / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": data_name(args),
        "config": {"workload": workload_name(args), "ticks_per_step": TICKS_PER_STEP,
                   "implementation": "reference tick compiled for the host CPU"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": used, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cuda_build": reference_cuda_time(args, snap, ctl),
    }
    print(json.dumps(line), flush=True)


def reference_cuda_time(args, snapshot, controls) -> dict | None:
    """The reference's own CUDA build (compiled from its sources for sm_100a),
    stepped through its RLEnvironment::step path with direct controls on the
    same states and the same control sequence as the b200 arm; device time
    from CUDA events around each step's ticks."""
    try:
        import torch

        if not torch.cuda.is_available():
            return None
        from oracle.refenv import RefGpu
    except Exception as exc:  # the CUDA build is optional for the CPU reference arm
        return {"unavailable": str(exc)}
    n_cars = args.blue + args.orange
    ref = RefGpu(args.n_sim, args.blue, args.orange, args.seed)
    ref.restore(snapshot)
    for i in range(args.warmup):
        ref.ticks(2, controls[i % len(controls)], TICKS_PER_STEP)
    total = 0.0
    for i in range(args.steps):
        total += ref.time_ticks(2, controls[(args.warmup + i) % len(controls)], TICKS_PER_STEP)
    ref.close()
    return {"value": args.n_sim * n_cars * TICKS_PER_STEP * args.steps / (total / 1e3), "unit": UNIT,
            "ms_per_step": total / args.steps, "steps": args.steps, "warmup": args.warmup,
            "what": "reference CUDA build (its sources, nvcc sm_100a --fmad=false -rdc), same states and controls"}


def stage_pass(env, step, first: int, count: int) -> tuple[dict, dict]:
    """Untimed pass with stage timing on: mean stage kernel ms (first sim slice,
    last tick of each step) and mean work-list sizes (all slices)."""
    env.set_stage_timing(True)
    times: dict[str, list[float]] = {}
    work: dict[str, list[int]] = {}
    for i in range(count):
        step(first + i)
        env.synchronize()
        for k, v in env.stage_times().items():
            times.setdefault(k, []).append(v)
        for k, v in env.stage_work().items():
            work.setdefault(k, []).append(v)
    env.set_stage_timing(False)
    return ({k: sum(v) / len(v) for k, v in times.items()}, {k: sum(v) / len(v) for k, v in work.items()})


def run_b200(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    from carl_b200 import capi

    device = local_rank
    torch.cuda.set_device(device)
    dev = torch.device("cuda", device)
    n_cars = args.blue + args.orange
    n_total_cars = args.n_sim * n_cars

    env = make_env(args, rank, device)
    stream = torch.cuda.ExternalStream(env.stream, device=dev)
    pool_n = max(4, min(16, args.steps + args.warmup))
    host_ctl = control_pool(n_total_cars, pool_n, args.seed + 1 + 7919 * rank)
    dev_ctl = [torch.from_numpy(c.view(np.int32)).to(dev) for c in host_ctl]
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def step(i):
        env.ticks(capi.ACTIONS_DIRECT, dev_ctl[i % pool_n], TICKS_PER_STEP)

    snap0 = env.snapshot() if rank == 0 and not args.no_cpu_baseline and world == 1 else None

    # ---- warm-up ----
    for i in range(args.warmup):
        step(i)
    env.synchronize()
    # The end-to-end pass replays the timed steps from this state, so both numbers
    # cover the same steps of the trajectory.
    snap_timed = None if args.no_e2e else env.snapshot()

    # ---- timed region: K steps enqueued back to back ----
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    enqueue_s = []
    sampler = ClockSampler(list(range(world))) if local_rank == 0 else None
    if sampler:
        sampler.start()
    barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        with torch.cuda.stream(stream):
            flush.fill_(i & 0xFF)
        h0 = time.perf_counter()
        starts[i].record(stream)
        step(args.warmup + i)
        ends[i].record(stream)
        enqueue_s.append(time.perf_counter() - h0)
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    barrier()
    clocks = sampler.stop() if sampler else None
    step_times = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    step_ms_rank = sum(step_times)
    ms_mine = env.last_tick_ms()  # device span of the last step's tick kernels

    # ---- stage times and work lists (untimed pass) ----
    stage_avg, work_avg = ({}, {}) if args.no_stages else stage_pass(env, step, args.warmup + args.steps,
                                                                         min(10, max(3, args.steps // 4)))

    # ---- per-rank record, gathered on every rank (same collective order everywhere) ----
    stage_names = list(capi.Env.STAGES)
    rec = [step_ms_rank, wall, 1e3 * statistics.mean(enqueue_s), 1e3 * max(enqueue_s), max(step_times),
           min(step_times), ms_mine] + [stage_avg.get(k, 0.0) for k in stage_names]
    t = torch.tensor(rec, dtype=torch.float64, device=dev)
    if world > 1:
        gathered = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        rows = [g.tolist() for g in gathered]
    else:
        rows = [t.tolist()]
    step_ms = max(r[0] for r in rows)
    per_rank = [{"rank": r, "ms_per_step": row[0] / args.steps, "wall_s": row[1], "enqueue_ms_mean": row[2],
                 "enqueue_ms_max": row[3], "step_ms_max": row[4], "step_ms_min": row[5],
                 "stage_ms": {k: round(v, 4) for k, v in zip(stage_names, row[7:]) if v}}
                for r, row in enumerate(rows)]

    agent_ticks_rank = n_total_cars * TICKS_PER_STEP * args.steps
    value = agent_ticks_rank * world / (step_ms / 1e3)

    # ---- end to end through the C ABI with host buffers ----
    e2e = None
    if not args.no_e2e:
        pinned_ctl = [torch.from_numpy(c).pin_memory() for c in host_ctl]
        rewards = torch.empty(args.n_sim, dtype=torch.float32).pin_memory()
        for i in range(min(args.warmup, 3)):  # warms the host-input graphs; the state is restored below
            env.ticks_host(capi.ACTIONS_DIRECT, pinned_ctl[i % pool_n].numpy(), TICKS_PER_STEP, rewards.numpy())
        env.restore(snap_timed)
        e_steps = max(1, min(args.steps, 50))
        e0 = [torch.cuda.Event(enable_timing=True) for _ in range(e_steps)]
        e1 = [torch.cuda.Event(enable_timing=True) for _ in range(e_steps)]
        barrier()
        torch.cuda.synchronize()
        for i in range(e_steps):
            with torch.cuda.stream(stream):
                flush.fill_(i & 0xFF)
                e0[i].record(stream)
            env.ticks_host(capi.ACTIONS_DIRECT, pinned_ctl[(args.warmup + i) % pool_n].numpy(), TICKS_PER_STEP,
                           rewards.numpy())
            e1[i].record(stream)
        torch.cuda.synchronize()
        barrier()
        ems = torch.tensor([sum(a.elapsed_time(b) for a, b in zip(e0, e1))], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e2e = {"value": n_total_cars * TICKS_PER_STEP * e_steps * world / (float(ems[0]) / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int(host_ctl[0].nbytes), "d2h_bytes_per_step": int(rewards.numel() * 4),
               "steps": e_steps, "path": "carlb_ticks_host (pinned host controls in, host rewards out)",
               "trajectory": "the timed steps replayed from the post-warm-up state with the same controls"}

    if rank != 0:
        env.close()
        return

    # ---- rooflines: whole tick from the event-timed step, and every stage kernel ----
    peak, peak_kind = measured_hbm_peak()
    bpat = bytes_per_agent_tick(n_cars)
    tick_ms = step_ms / args.steps / TICKS_PER_STEP
    tick_achieved = bpat * n_total_cars / (tick_ms / 1e3) / 1e9
    roofline_tick = {"bound": "hbm", "achieved": tick_achieved, "peak": peak, "unit": "GB/s",
                     "frac": tick_achieved / peak, "model": "CARLB-v1", "bytes_per_agent_tick": bpat,
                     "tick_ms": tick_ms, "tick_ms_source": "event-timed step (max over ranks) / 8"}
    flops = fp32_flops_per_car_tick()
    roofline_fp32 = None
    if flops:
        sm_max = float((clocks or {}).get("sm_max_mhz") or 1965.0)
        fp32_peak = 148 * 128 * 2 * sm_max * 1e6 / 1e12
        fp32_achieved = flops * n_total_cars / (tick_ms / 1e3) / 1e12
        roofline_fp32 = {"bound": "fp32", "achieved": fp32_achieved, "peak": fp32_peak, "unit": "TFLOP/s",
                         "frac": fp32_achieved / fp32_peak, "flop_per_car_tick": flops,
                         "peak_kind": "nominal: 148 SMs x 128 FP32 lanes x 2 FLOP x max SM clock"}
    roofline = None
    if stage_avg:
        # A stage kernel launch covers one sim slice (the timed one is slice 0);
        # work lists are summed over slices, so one slice gets its share.
        groups = world_groups(args)
        slice_cars, slice_sims = n_total_cars / groups, args.n_sim / groups
        slice_work = {k: v / groups for k, v in work_avg.items()}
        per_stage = {}
        for k, ms in stage_avg.items():
            b = stage_bytes(k, slice_cars, slice_sims, slice_work)
            per_stage[k] = {"ms": round(ms, 4), "algorithmic_bytes": b,
                            "achieved_gbs": round(b / (ms / 1e3) / 1e9, 2), "frac": b / (ms / 1e3) / 1e9 / peak}
        dom = max(stage_avg, key=stage_avg.get)
        d = per_stage[dom]
        roofline = {"bound": "hbm", "achieved": d["achieved_gbs"], "peak": peak, "unit": "GB/s", "frac": d["frac"],
                    "traffic": traffic_per_launch(dom, args.n_sim), "peak_kind": peak_kind, "kernel": dom + "Kernel",
                    "launch_ms": d["ms"], "algorithmic_bytes_per_launch": d["algorithmic_bytes"],
                    "sim_slices": groups, "selection": "the stage kernel with the longest mean duration",
                    "stages": per_stage, "work_lists_per_tick": {k: round(v, 1) for k, v in work_avg.items()}}

    cpu = None
    if snap0 is not None:
        secs_target = 12.0
        threads = host_threads()
        v, secs, used = reference_cpu_time(snap0, args.n_sim, args.blue, args.orange, args.seed, host_ctl, 1, threads)
        more = int(max(0, min(16, secs_target / max(secs, 1e-3) - 1)))
        steps_done, secs_tot = 1, secs
        if more:
            v, secs_tot, used = reference_cpu_time(snap0, args.n_sim, args.blue, args.orange, args.seed, host_ctl, more,
                                                   threads)
            steps_done = more
        cpu = {"value": v, "unit": UNIT, "cores": used, "kind": "reference",
               "sample": f"{steps_done} steps x {TICKS_PER_STEP} ticks of the same {args.blue}v{args.orange} "
                         f"n_sim={args.n_sim} workload ({secs_tot:.1f} s) with the reference tick compiled for the "
                         f"host, OpenMP over sims"}

    line = {
        "metric": metric_name(args), "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": data_name(args),
        "config": {"workload": workload_name(args), "ticks_per_step": TICKS_PER_STEP,
                   "sims_total": args.n_sim * world, "parallelism": f"sim-sharded x{world}",
                   "compat_flags": 0, "semantics": "the reference's CUDA build (default mode)",
                   "l2": "256 MiB buffer written before each timed step", "wall_s": wall},
        "clocks": clocks, "e2e": e2e,
        "gpu_launches": args.steps * launches_per_step(world_groups(args)),
        "roofline": roofline, "roofline_tick": roofline_tick, "roofline_fp32": roofline_fp32, "cpu_baseline": cpu,
        "per_rank": per_rank,
    }
    print(json.dumps(line), flush=True)
    env.close()


RESET_FRACTION = 0.01


def kickoff_rows(n_sim: int, nb: int, no: int, seed: int) -> dict:
    """apply_reset_state inputs, one row per sim, holding each sim's kickoff state."""
    from carl_b200 import capi

    n_cars = nb + no
    env = capi.Env(n_sim, nb, no, seed)
    env.reset()
    f = lambda name: env.read_field(name).view(np.float32)  # noqa: E731
    rows = {
        "ball_position": f("BALL_POS").reshape(n_sim, 3), "ball_velocity": f("BALL_VEL").reshape(n_sim, 3),
        "ball_angular_velocity": f("BALL_ANG").reshape(n_sim, 3),
        "car_position": f("CAR_POS").reshape(n_sim, n_cars, 3), "car_rotation": f("CAR_ROT").reshape(n_sim, n_cars, 4),
        "car_velocity": f("CAR_VEL").reshape(n_sim, n_cars, 3),
        "car_angular_velocity": f("CAR_ANG").reshape(n_sim, n_cars, 3),
        "car_demoed": env.read_field("CAR_IS_DEMOED").reshape(n_sim, n_cars).astype(np.uint8),
        "blue_score": np.zeros(n_sim, np.int32), "orange_score": np.zeros(n_sim, np.int32),
        "episode_ticks": np.zeros(n_sim, np.int32),
    }
    env.close()
    return {k: np.ascontiguousarray(v) for k, v in rows.items()}


class _ArrayInterface:
    """A float32 device buffer of the env described for torch.as_tensor."""

    def __init__(self, ptr: int, shape: tuple):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": "<f4",
                                         "strides": None, "version": 3, "stream": None}


def device_view(env, which: int, torch):
    """Zero-copy torch view of an env output buffer (float32)."""
    ptr, shape, _ = env.buffer(which)
    return torch.as_tensor(_ArrayInterface(ptr, shape), device=torch.device("cuda", torch.cuda.current_device()))


def run_env_workload(args, resets: bool, rank: int = 0, world: int = 1, local_rank: int = 0) -> None:
    """The env step path (python/carl.cu:312-370: frameskip ticks, then reward /
    done / transition packing, auto-reset and obs / state packing), timed with
    CUDA events on the env stream, beside the same sequence on the reference's
    own CUDA build (`carlrefgpu_time_reset_steps`, rank 0 only).

    step:  config C3 (3v3, n_sim sims, seeded floor states), frameskip 8 (the
           gymnasium wrapper's default), discrete actions; env-steps/s.  Team
           sizes, sims and frameskip follow --blue/--orange/--n-sim/--frameskip
           (C2: 1v1, 65536 sims, frameskip 1, so obs are packed every tick).
    c5:    config C5 (4v4, --reset-n-sim sims per GPU, C4 mixed states),
           frameskip 1, each env step followed by a masked apply_reset_state
           that puts a random 1 % of the sims back to their kickoff state, and
           the obs handed to torch (torch's stream waits for the env stream,
           reads the obs, and the env stream waits for torch before the next
           step, as the gymnasium wrapper's _sync does).  Every rank steps its
           own shard (global sim offset rank * n_sim); the value is the whole
           job's agent-steps/s from the maximum over ranks of the timed steps.
           On one GPU the separate reset part kernels (CARLB_FUSED_RESET=0)
           run the same sequence as a second mode."""
    import torch
    import torch.distributed as dist

    from carl_b200 import capi, workloads

    torch.cuda.set_device(local_rank)
    if resets:
        nb = no = 4
        n_sim, frameskip = args.reset_n_sim, 1
    else:
        nb, no = args.blue, args.orange
        n_sim, frameskip = args.n_sim, args.frameskip
    n_cars = nb + no
    rng = np.random.default_rng(args.seed + 5 + 7919 * rank)
    rows = kickoff_rows(n_sim, nb, no, args.seed) if resets else None
    n_steps = args.warmup + args.steps
    masks = (rng.uniform(size=(n_steps, n_sim)) < RESET_FRACTION).astype(np.uint8) if resets else None
    actions = workloads.discrete_actions(rng, n_sim * n_cars).reshape(n_sim, n_cars, 7)
    order = ["ball_position", "ball_velocity", "ball_angular_velocity", "car_position", "car_rotation",
             "car_velocity", "car_angular_velocity", "car_demoed"]
    results = {}
    snap = None
    modes = ("fused", "parts") if resets and world == 1 else (("fused",) if resets else ("b200",))
    for mode in modes:
        os.environ["CARLB_FUSED_RESET"] = "0" if mode == "parts" else "1"
        env = capi.Env(n_sim, nb, no, args.seed, frameskip=frameskip, device=local_rank, sim_offset=rank * n_sim)
        if snap is None:
            (workloads.mixed_state if resets else workloads.floor_state)(env, args.seed + 1000 * rank)
            snap = env.snapshot()
        else:
            env.restore(snap)
        stream = torch.cuda.ExternalStream(env.stream)
        dev = {k: torch.from_numpy(v).cuda() for k, v in rows.items()} if resets else {}
        dmask = torch.from_numpy(masks).cuda() if resets else None
        act = torch.from_numpy(actions).cuda()
        obs_view = device_view(env, capi.BUF_OBS, torch) if resets else None
        seen = torch.zeros((), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
        current = torch.cuda.current_stream()
        for i in range(n_steps):
            timed = i >= args.warmup
            e = ev[i - args.warmup] if timed else None
            if timed:
                e[0].record(stream)
            env.env_step(capi.ACTIONS_DISCRETE, act)
            if timed:
                e[1].record(stream)
            if resets:
                env.apply_reset_state(n_sim, *[dev[o] for o in order], True, None, None, dev["blue_score"],
                                      dev["orange_score"], dev["episode_ticks"], reset_mask=dmask[i])
                if timed:
                    e[2].record(stream)
                # Stream handoff of the obs to torch, and back.
                current.wait_stream(stream)
                seen += obs_view[:, :, 0].sum()
                stream.wait_stream(current)
                if timed:
                    e[3].record(stream)
        env.synchronize()
        torch.cuda.synchronize()
        step_ms = sum(a.elapsed_time(b) for a, b, _, _ in ev) / args.steps
        reset_ms = sum(b.elapsed_time(c) for _, b, c, _ in ev) / args.steps if resets else 0.0
        handoff_ms = sum(c.elapsed_time(d) for _, _, c, d in ev) / args.steps if resets else 0.0
        t = torch.tensor([step_ms, reset_ms, handoff_ms], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        results[mode] = {"step_ms": float(t[0]), "reset_ms": float(t[1]), "handoff_ms": float(t[2])}
        env.close()
    os.environ.pop("CARLB_FUSED_RESET", None)
    if rank == 0:
        try:
            from oracle.refenv import RefGpu

            ref = RefGpu(n_sim, nb, no, args.seed, frameskip=frameskip)
            ref.restore(snap)
            if args.warmup:
                ref.time_reset_steps(capi.ACTIONS_DISCRETE, actions, args.warmup, rows,
                                     masks[: args.warmup] if resets else None)
            s_ms, r_ms = ref.time_reset_steps(capi.ACTIONS_DISCRETE, actions, args.steps, rows,
                                              masks[args.warmup:] if resets else None)
            ref.close()
            results["reference_cuda_build"] = {"step_ms": s_ms / args.steps, "reset_ms": r_ms / args.steps,
                                               "handoff_ms": 0.0, "n_gpus": 1}
        except Exception as exc:  # the reference build is optional here
            results["reference_cuda_build"] = {"unavailable": str(exc)}
    if rank != 0:
        return
    for name, r in results.items():
        if "step_ms" in r:
            ms = r["step_ms"] + r["reset_ms"] + r["handoff_ms"]
            gpus = r.get("n_gpus", world)
            r["agent_steps_per_s"] = n_sim * n_cars * frameskip * gpus / (ms / 1e3)
            r["env_steps_per_s"] = n_sim * gpus / (ms / 1e3)
    ours = results["fused" if resets else "b200"]
    if resets:
        metric = "agent-steps/sec, env steps with 1% masked resets per step and obs handed to torch (C5)"
        workload = (f"C5 4v4 n_sim={n_sim} per GPU ({n_sim * world} total), frameskip 1, env_step + masked "
                    f"apply_reset_state of {RESET_FRACTION:.0%} of sims per step + obs stream handoff to torch")
        data = "synthetic (seeded C4 mixed states, discrete actions, random 1% masks, kickoff reset rows)"
    else:
        metric = f"env-steps/sec at {nb}v{no} n_sim={n_sim}, frameskip {frameskip}"
        name = "C2" if (nb, no, frameskip) == (1, 1, 1) else "C3"
        workload = f"{name} {nb}v{no} n_sim={n_sim}, env_step (frameskip {frameskip} ticks + packing), discrete actions"
        data = "synthetic (seeded floor states, discrete actions)"
    line = {
        "metric": metric, "value": ours["agent_steps_per_s"] if resets else ours["env_steps_per_s"],
        "unit": UNIT if resets else "env-steps/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ours["step_ms"] + ours["reset_ms"] + ours["handoff_ms"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": data,
        "config": {"workload": workload, "compat_flags": 0}, "modes": results,
    }
    if resets:
        line["gpu_launches_per_reset"] = {"fused": 1, "parts": 8}
    print(json.dumps(line), flush=True)


def reference_action_mask(observation, previous_controls: bool):
    """The reference's own mask (python/carl/gymnasium/action.py:17-37), the torch
    op chain the device kernel replaces; timed as that row's reference arm."""
    import torch as th

    from carl_b200 import carl

    size = carl.OBS_PREVIOUS_CONTROLS if previous_controls else 0
    on_ground = observation[..., carl.OBS_EGO_ON_GROUND_INDEX].bool()
    has_boost = observation[..., carl.OBS_EGO_BOOST_INDEX].gt(0)
    flip_available = observation[..., carl.OBS_EGO_FLIP_INDEX - size].bool()
    jump_available = on_ground | (flip_available & (observation[..., carl.OBS_EGO_DODGE_TIME_INDEX - size] > carl.PHYS_DT))
    mask = th.ones((*observation.shape[:-1], carl.ACTION_LOGITS), dtype=th.bool, device=observation.device)
    mask[..., carl.ACTION_POWERSLIDE_LOGIT] = on_ground
    mask[..., carl.ACTION_BOOST_LOGIT] = has_boost
    mask[..., carl.ACTION_JUMP_LOGIT] = jump_available
    return mask


def run_mask_workload(args) -> None:
    """Action masks of a packed observation batch (config C5's per-GPU shard:
    4v4, --reset-n-sim sims): the device kernel (carl_b200.action.CARLActionCodec)
    against the reference's torch op chain, both on torch's current stream,
    CUDA-event timed, results checked equal."""
    import torch

    from carl_b200 import carl, workloads
    from carl_b200.action import CARLActionCodec

    n_sim = args.reset_n_sim
    env = carl.Env(n_sim, 4, 4, args.seed)
    workloads.mixed_state(env._env, args.seed)
    rng = np.random.default_rng(args.seed + 9)
    obs = env.step(torch.from_numpy(workloads.discrete_actions(rng, n_sim * 8).reshape(n_sim, 8, 7)).cuda())
    torch.cuda.current_stream().wait_stream(torch.cuda.ExternalStream(env.stream))
    codec = CARLActionCodec()
    assert torch.equal(codec.mask(obs), reference_action_mask(obs, False))
    out = {}
    for name, fn in (("b200", codec.mask), ("reference_torch", lambda o: reference_action_mask(o, False))):
        for _ in range(args.warmup):
            fn(obs)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            fn(obs)
        end.record()
        end.synchronize()
        out[name] = {"ms": start.elapsed_time(end) / args.steps}
    rows = n_sim * 8
    for r in out.values():
        r["rows_per_s"] = rows / (r["ms"] / 1e3)
    line = {
        "metric": "action-mask rows/sec", "value": out["b200"]["rows_per_s"], "unit": "rows/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": out["b200"]["ms"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (obs packed from seeded C4 mixed states after one env step)",
        "config": {"workload": f"CARLActionCodec.mask of [{n_sim}, 8, {obs.shape[-1]}] observations (C5 shard)"},
        "modes": out,
    }
    print(json.dumps(line), flush=True)
    env.close()


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload in ("step", "mask") or (args.workload == "c5" and args.impl == "reference"):
        if rank == 0:
            (run_mask_workload(args) if args.workload == "mask"
             else run_env_workload(args, resets=args.workload == "c5"))
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "c5":
            run_env_workload(args, True, rank, world, local_rank)
        else:
            run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
