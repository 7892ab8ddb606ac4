"""Throughput benchmark of the batched Rocket League tick on B200.

Workload (config C3): 3v3, n_sim = 32768 sims per GPU, default arena, seeded
synthetic initial states (cars uniform over the field floor, planar velocity
N(0, 800 uu/s), yaw uniform, boost U[0, 100], ball at rest at centre) and
direct controls redrawn every 8 ticks (throttle/steer/pitch/yaw/roll U[-1, 1],
jump/boost/handbrake Bernoulli(0.3)).

A *step* is one control period: the controls for all cars are staged and 8
physics ticks run (one launch of the fused tick kernel).  The metric is
agent-steps/s = cars x ticks / s, one agent-step being one car advanced one
120 Hz tick.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

For N > 1 it runs under torch.distributed.run, one rank per GPU; each rank
simulates its own contiguous slice of sims (global sim offset rank*n_sim), so
per-GPU work is fixed (weak scaling) and there is no collective in the tick.

Timed region: barrier + synchronize, K steps, synchronize + barrier.  Each
step's device time is taken with CUDA events on the env stream; between timed
steps a 256 MiB buffer is written to flush the 126 MB L2 (outside the events).
The roofline uses the event-timed duration of the dominant stage kernel (CUDA
events around each stage kernel of the first sim slice, last tick of each step),
and a second figure covers the whole tick.
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
# Algorithmic bytes of single stage kernels, per car and per sim of one tick:
# the words the stage must read and write (arena tables are L2-resident and
# excluded).  flat: pose in (pos, vel, ang, cen, rot: 16 words), candidate
# list start, count, SAT hit mask (9 words) and ray keys (8 words) out, episode
# tick read-modify-write per sim.  rayCtl: pose, keys, controls state in
# (74 words), rays, wheel bits and controls state out (62 words), ball position
# per sim.  susp: hits, rays, body, suspension, friction and manifold state in
# (70 words), suspension state, friction and velocities out (33 words).
# ballPrep: ball state in (22 words), hand-over values out (15 words).
STAGE_BYTES = {
    "flat": (140, 8),
    "rayCtl": (544, 12),
    "susp": (412, 0),
    "ballPrep": (0, 148),
}
METRIC = "agent-steps/sec at 3v3 n_sim=32768"
UNIT = "agent-steps/s"


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
    ap.add_argument("--workload", choices=["c3", "step", "reset", "mask"], default="c3",
                    help="c3: the headline tick throughput; step: env steps at frameskip 8 (ticks + packing); "
                         "reset: env steps with masked resets (C5 shard); mask: device action masks")
    ap.add_argument("--reset-n-sim", type=int, default=131072, help="sims of the reset workload (4v4)")
    ap.add_argument("--frameskip", type=int, default=TICKS_PER_STEP,
                    help="ticks per env step of the step workload (1 with --blue 1 --orange 1 --n-sim 65536: "
                         "config C2, obs packed every tick)")
    return ap.parse_args()


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, device: int):
        self.bus_id = ""
        try:
            import torch

            pr = torch.cuda.get_device_properties(device)
            self.bus_id = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
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
            if self.bus_id and f[1].lower()[-12:] != self.bus_id[-12:]:
                continue
            rows.append(f)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        reasons = sorted({name for r in rows for name, v in zip(self.REASONS, r[6:10]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------ workload ----
def make_env(args, rank: int, device: int):
    from carl_b200 import capi, workloads

    env = capi.Env(args.n_sim, args.blue, args.orange, seed=args.seed, device=device,
                   sim_offset=rank * args.n_sim)
    workloads.floor_state(env, args.seed + 1000 * rank)
    return env


def control_pool(n_cars_total: int, count: int, seed: int):
    from carl_b200 import workloads

    rng = np.random.default_rng(seed)
    return [workloads.controls(rng, n_cars_total) for _ in range(count)]


def traffic_per_launch(stage: str, n_sim: int) -> float | None:
    """DRAM bytes per launch of a stage kernel, from the committed ncu summary
    of the staged tick (stated for n_sim = 32768, 2 slices; traffic grows with
    the sims, so it is scaled to this run's n_sim).  None when not captured."""
    path = ROOT / "profiles" / "staged_tick_3v3_32768.md"
    if not path.exists():
        return None
    key = f"traffic_bytes_per_launch[{stage}]:"
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
    """The reference arm: the reference's own CPU tick on the host cores."""
    if rank != 0:
        return
    from carl_b200 import capi, workloads

    n_cars = args.blue + args.orange
    # The initial state is built on the host restatement of the reference so the
    # arm needs no GPU: kickoff reset, then the same seeded floor distribution.
    from oracle.refenv import RefCpu

    threads = host_threads()
    RefCpu.set_threads(threads)
    ref = RefCpu(args.n_sim, args.blue, args.orange, args.seed)
    workloads.floor_state(ref, args.seed)
    snap = ref.snapshot()
    ref.close()
    pool_n = max(4, min(16, args.steps + args.warmup))
    ctl = control_pool(args.n_sim * n_cars, pool_n, args.seed + 1)
    steps = max(1, min(args.steps, 8))
    warm = max(0, min(args.warmup, 1))
    if warm:
        reference_cpu_time(snap, args.n_sim, args.blue, args.orange, args.seed, ctl, warm, threads)
    value, secs, used = reference_cpu_time(snap, args.n_sim, args.blue, args.orange, args.seed, ctl, steps, threads)
    sample = (f"{steps} steps x {TICKS_PER_STEP} ticks of the full 3v3 n_sim={args.n_sim} workload "
              f"({secs:.1f} s), OpenMP over sims")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": secs * 1e3 / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded C3 floor states, direct controls)",
        "config": {"workload": f"C3 {args.blue}v{args.orange} n_sim={args.n_sim}, direct controls held 8 ticks",
                   "ticks_per_step": TICKS_PER_STEP, "implementation": "reference tick compiled for the host CPU"},
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

    # ---- timed region ----
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kernel_ms = []
    stage_ms: dict[str, list[float]] = {}
    try:
        env.set_stage_timing(True)
        staged = True
    except capi.CarlbError:  # the fused path (CARLB_TICK_PATH=fused) has one kernel per launch
        staged = False
    sampler = ClockSampler(device)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        with torch.cuda.stream(stream):
            flush.fill_(i & 0xFF)
            starts[i].record(stream)
        step(args.warmup + i)
        ends[i].record(stream)
        env.synchronize()
        kernel_ms.append(env.last_tick_ms())
        if staged:
            for name, ms in env.stage_times().items():
                stage_ms.setdefault(name, []).append(ms)
    torch.cuda.synchronize()
    barrier()
    wall = time.perf_counter() - wall0
    clocks = sampler.stop()
    step_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    kern_ms = sum(kernel_ms)

    t = torch.tensor([step_ms, kern_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms, kern_ms = float(t[0]), float(t[1])
    if staged:
        env.set_stage_timing(False)
    stage_avg = {k: sum(v) / len(v) for k, v in stage_ms.items()}

    agent_ticks_rank = n_total_cars * TICKS_PER_STEP * args.steps
    value = agent_ticks_rank * world / (step_ms / 1e3)

    # ---- end to end through the C ABI with host buffers ----
    e2e = None
    if not args.no_e2e:
        pinned_ctl = [torch.from_numpy(c).pin_memory() for c in host_ctl[: min(pool_n, 8)]]
        rewards = torch.empty(args.n_sim, dtype=torch.float32).pin_memory()
        for i in range(min(args.warmup, 3)):
            env.ticks_host(capi.ACTIONS_DIRECT, pinned_ctl[i % len(pinned_ctl)].numpy(), TICKS_PER_STEP, rewards.numpy())
        e_steps = max(1, min(args.steps, 50))
        e0 = [torch.cuda.Event(enable_timing=True) for _ in range(e_steps)]
        e1 = [torch.cuda.Event(enable_timing=True) for _ in range(e_steps)]
        barrier()
        torch.cuda.synchronize()
        for i in range(e_steps):
            with torch.cuda.stream(stream):
                flush.fill_(i & 0xFF)
                e0[i].record(stream)
            env.ticks_host(capi.ACTIONS_DIRECT, pinned_ctl[i % len(pinned_ctl)].numpy(), TICKS_PER_STEP, rewards.numpy())
            e1[i].record(stream)
        torch.cuda.synchronize()
        barrier()
        ems = torch.tensor([sum(a.elapsed_time(b) for a, b in zip(e0, e1))], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e2e = {"value": n_total_cars * TICKS_PER_STEP * e_steps * world / (float(ems[0]) / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int(host_ctl[0].nbytes), "d2h_bytes_per_step": int(rewards.numel() * 4),
               "steps": e_steps, "path": "carlb_ticks_host (pinned host controls in, host rewards out)"}

    if rank != 0:
        env.close()
        return

    # ---- roofline of the dominant stage kernel, and of the whole tick ----
    peak, peak_kind = measured_hbm_peak()
    bpat = bytes_per_agent_tick(n_cars)
    tick_ms = kern_ms / args.steps / TICKS_PER_STEP
    tick_achieved = bpat * n_total_cars / (tick_ms / 1e3) / 1e9
    roofline_tick = {"bound": "hbm", "achieved": tick_achieved, "peak": peak, "unit": "GB/s",
                     "frac": tick_achieved / peak, "model": "CARLB-v1", "bytes_per_agent_tick": bpat,
                     "tick_ms": tick_ms}
    # FP32 SIMT roof of the whole tick: counted FLOPs per car-tick (ncu summary)
    # over the nominal FP32 peak at the sampled maximum SM clock.
    flops = fp32_flops_per_car_tick()
    roofline_fp32 = None
    if flops:
        sm_max = float(clocks.get("sm_max_mhz") or 1965.0)
        fp32_peak = 148 * 128 * 2 * sm_max * 1e6 / 1e12
        fp32_achieved = flops * n_total_cars / (tick_ms / 1e3) / 1e12
        roofline_fp32 = {"bound": "fp32", "achieved": fp32_achieved, "peak": fp32_peak, "unit": "TFLOP/s",
                         "frac": fp32_achieved / fp32_peak, "flop_per_car_tick": flops,
                         "peak_kind": "nominal: 148 SMs x 128 FP32 lanes x 2 FLOP x max SM clock"}
    if staged:
        # A stage kernel launch covers one sim slice (the timed one is slice 0).
        groups = world_groups(args)
        modelled = {k: v for k, v in stage_avg.items() if k in STAGE_BYTES}
        dom = max(modelled, key=modelled.get)
        per_car, per_sim = STAGE_BYTES[dom]
        dom_bytes = (per_car * n_total_cars + per_sim * args.n_sim) / groups
        dom_ms = stage_avg[dom]
        achieved = dom_bytes / (dom_ms / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                    "traffic": traffic_per_launch(dom, args.n_sim), "peak_kind": peak_kind, "kernel": dom + "Kernel",
                    "launch_ms": dom_ms, "algorithmic_bytes_per_launch": dom_bytes, "sim_slices": groups,
                    "stage_ms": {k: round(v, 4) for k, v in stage_avg.items()},
                    "largest_stage": max(stage_avg, key=stage_avg.get)}
    else:
        roofline = dict(roofline_tick, kernel="tickKernel (fused, 8 ticks per launch)", peak_kind=peak_kind,
                        traffic=None, launch_ms=kern_ms / args.steps)

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
               "sample": f"{steps_done} steps x {TICKS_PER_STEP} ticks of the same 3v3 n_sim={args.n_sim} workload "
                         f"({secs_tot:.1f} s) with the reference tick compiled for the host, OpenMP over sims"}

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded C3 floor states, direct controls redrawn every 8 ticks)",
        "config": {"workload": f"C3 {args.blue}v{args.orange} n_sim={args.n_sim} per GPU, direct controls held 8 ticks",
                   "ticks_per_step": TICKS_PER_STEP, "sims_total": args.n_sim * world,
                   "parallelism": f"sim-sharded x{world}", "l2": "256 MiB buffer written between timed steps",
                   "wall_s": wall},
        "clocks": clocks, "e2e": e2e,
        "gpu_launches": args.steps * (launches_per_step(world_groups(args)) if staged else 1),
        "roofline": roofline, "roofline_tick": roofline_tick, "roofline_fp32": roofline_fp32, "cpu_baseline": cpu,
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


def run_env_workload(args, resets: bool) -> None:
    """The env step path (python/carl.cu:312-370: frameskip ticks, then reward /
    done / transition packing, auto-reset and obs / state packing), timed with
    CUDA events on the env stream, beside the same sequence on the reference's
    own CUDA build (`carlrefgpu_time_reset_steps`).

    step:  config C3 (3v3, n_sim sims, seeded floor states), frameskip 8 (the
           gymnasium wrapper's default), discrete actions; env-steps/s.  Team
           sizes, sims and frameskip follow --blue/--orange/--n-sim/--frameskip
           (C2: 1v1, 65536 sims, frameskip 1, so obs are packed every tick).
    reset: config C5's per-GPU shard (4v4, --reset-n-sim sims, C4 mixed states),
           frameskip 1, each env step followed by a masked apply_reset_state
           that puts a random 1 % of the sims back to their kickoff state; the
           fused reset kernel, the separate part kernels (CARLB_FUSED_RESET=0)
           and the reference run the same sequence, step and reset timed apart."""
    import torch

    from carl_b200 import capi, workloads

    if resets:
        nb = no = 4
        n_sim, frameskip = args.reset_n_sim, 1
    else:
        nb, no = args.blue, args.orange
        n_sim, frameskip = args.n_sim, args.frameskip
    n_cars = nb + no
    rng = np.random.default_rng(args.seed + 5)
    rows = kickoff_rows(n_sim, nb, no, args.seed) if resets else None
    n_steps = args.warmup + args.steps
    masks = (rng.uniform(size=(n_steps, n_sim)) < RESET_FRACTION).astype(np.uint8) if resets else None
    actions = workloads.discrete_actions(rng, n_sim * n_cars).reshape(n_sim, n_cars, 7)
    order = ["ball_position", "ball_velocity", "ball_angular_velocity", "car_position", "car_rotation",
             "car_velocity", "car_angular_velocity", "car_demoed"]
    results = {}
    snap = None
    for mode in (("fused", "parts") if resets else ("b200",)):
        os.environ["CARLB_FUSED_RESET"] = "0" if mode == "parts" else "1"
        env = capi.Env(n_sim, nb, no, args.seed, frameskip=frameskip)
        if snap is None:
            (workloads.mixed_state if resets else workloads.floor_state)(env, args.seed)
            snap = env.snapshot()
        else:
            env.restore(snap)
        stream = torch.cuda.ExternalStream(env.stream)
        dev = {k: torch.from_numpy(v).cuda() for k, v in rows.items()} if resets else {}
        dmask = torch.from_numpy(masks).cuda() if resets else None
        act = torch.from_numpy(actions).cuda()
        torch.cuda.synchronize()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
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
        env.synchronize()
        step_ms = sum(a.elapsed_time(b) for a, b, _ in ev) / args.steps
        reset_ms = sum(b.elapsed_time(c) for _, b, c in ev) / args.steps
        results[mode] = {"step_ms": step_ms, "reset_ms": reset_ms}
        env.close()
    os.environ.pop("CARLB_FUSED_RESET", None)
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
        results["reference_cuda_build"] = {"step_ms": s_ms / args.steps, "reset_ms": r_ms / args.steps}
    except Exception as exc:  # the reference build is optional here
        results["reference_cuda_build"] = {"unavailable": str(exc)}
    for r in results.values():
        if "step_ms" in r:
            ms = r["step_ms"] + r["reset_ms"]
            r["agent_steps_per_s"] = n_sim * n_cars * frameskip / (ms / 1e3)
            r["env_steps_per_s"] = n_sim / (ms / 1e3)
    ours = results["fused" if resets else "b200"]
    if resets:
        metric = "agent-steps/sec, env steps with 1% masked resets per step"
        workload = (f"C5 per-GPU shard: 4v4 n_sim={n_sim}, frameskip 1, env_step + masked apply_reset_state "
                    f"of {RESET_FRACTION:.0%} of sims per step")
        data = "synthetic (seeded C4 mixed states, discrete actions, random 1% masks, kickoff reset rows)"
    else:
        metric = f"env-steps/sec at {nb}v{no} n_sim={n_sim}, frameskip {frameskip}"
        name = "C2" if (nb, no, frameskip) == (1, 1, 1) else "C3"
        workload = f"{name} {nb}v{no} n_sim={n_sim}, env_step (frameskip {frameskip} ticks + packing), discrete actions"
        data = "synthetic (seeded floor states, discrete actions)"
    line = {
        "metric": metric, "value": ours["agent_steps_per_s"] if resets else ours["env_steps_per_s"],
        "unit": UNIT if resets else "env-steps/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ours["step_ms"] + ours["reset_ms"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": data, "config": {"workload": workload},
        "modes": results,
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
    if args.workload in ("reset", "step"):
        if rank == 0:
            run_env_workload(args, resets=args.workload == "reset")
        return
    if args.workload == "mask":
        if rank == 0:
            run_mask_workload(args)
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
        run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
