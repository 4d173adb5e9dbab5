"""world-steps/s of the batched Box2D step on B200 (BASELINE.json's metric), one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1] [--worlds 4096] [--impl ours|reference]

Workload: BASELINE.json configs[1] (the character rig: pot, hub and bullet hammer on a revolute motor and a
prismatic slide, over a 2000-segment chain level with 60 rocks), polygon-terrain variant (the reference engine has
no edge/chain shapes), seeded synthetic worlds (goib2d/configs.py), 4096 worlds per GPU, dt 0.02, 8/3 iterations,
continuous physics on. A bench step = one call of the public step (goib2d_step_seq) running --substeps (default 10)
b2World::Steps of every world in one persistent launch, each physics step with its own per-world action from a disc
of radius 2 driving the two joint motors; the value counts world-steps (worlds x physics steps). The first --skip
(default 100) physics steps of the episode run untimed before the warm-up, so that the timed steps lie in the
episode's steady part (c1's first ~50 steps, the rig falling onto the level, run faster than the rest). L2 is flushed
(a 256 MiB write) between timed calls; each call is timed with CUDA events on the launching stream and the K
durations are summed; max over ranks.

--impl reference: the reference engine's algorithm on the host cores - the parity oracle (oracle/, a C++
restatement of goi_jax/box2d, bit-identical to it on every golden vector) on all host threads, over a bounded sample
of the same workload. The reference's own JAX engine cannot run here (no jax/jaxlib in the image).
"""
import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "getting-over-it-rl_b200"))
sys.path.insert(0, str(ROOT / "tests"))

METRIC = "world-steps/sec"
UNIT = "world-steps/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c1", choices=("c0", "c1", "c2", "c3", "c4", "c0e", "c1e", "c3e", "c4e"))
    ap.add_argument("--worlds", type=int, default=None, help="worlds per GPU (default: the config's N)")
    ap.add_argument("--substeps", type=int, default=10,
                    help="physics steps per call (goib2d_step_seq: one launch, one row of actions per step)")
    ap.add_argument("--skip", type=int, default=100, help="untimed physics steps before the warm-up, so that the "
                                                           "timed steps lie in the episode's steady part")
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-sample-worlds", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def actions_for(n, steps, seed, first=0):
    """Per-world, per-step targets on a disc of radius 2, uniform in area (r = 2 sqrt(u), theta = 2 pi v)."""
    rng = np.random.default_rng([seed, 7, first])
    u, v = rng.uniform(0, 1, (steps, n)), rng.uniform(0, 1, (steps, n))
    r, th = 2.0 * np.sqrt(u), 2.0 * np.pi * v
    return np.stack([r * np.cos(th), r * np.sin(th)], -1).astype(np.float32)  # (steps, n, 2)


def state_bytes(state):
    """Algorithmic bytes of one world-step: the per-world State read once and written once (compact layout)."""
    from goib2d import native
    B, rows = state.bodies.type.shape[1], state.fixtures.friction.shape[1]
    J, C = state.joints.motor_speed.shape[1], state.contacts.pair.shape[1]
    return 2 * native.state_bytes_per_world(B, rows, J, C)


class Clocks:
    """The SM clock, its maximum and the active clock-event (throttle) reasons of the bench's GPU, read through NVML
    every 2 ms by a thread while the timed region runs (nvidia-smi's query when NVML is unavailable). Reads only."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, device):
        self.device, self.rows, self.thread, self.nvml, self.h = device, [], None, None, None

    def _handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.device)
        try:  # the same GPU as the CUDA device, whatever CUDA_VISIBLE_DEVICES maps
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(int(self.device))

    def start(self):
        import threading
        try:
            self.nvml, self.h = self._handle()
        except Exception:
            self.nvml = None
            return
        nv, h = self.nvml, self.h
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        self.stop_flag = False

        def poll():
            while not self.stop_flag:
                self.rows.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), int(get_reasons(h))))
                time.sleep(0.002)
        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()

    def stop(self):
        if self.nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["NVML unavailable"], "samples": 0}
        self.stop_flag = True
        self.thread.join(timeout=5)
        sm = [r[0] for r in self.rows]
        mask = 0
        for r in self.rows:
            mask |= r[1]
        mx = self.nvml.nvmlDeviceGetMaxClockInfo(self.h, self.nvml.NVML_CLOCK_SM)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": float(mx),
                "reasons": sorted(n for b, n in self.REASONS.items() if mask & b), "samples": len(sm),
                "source": "NVML, every 2 ms during the timed region"}


WORKLOADS = {
    "c0": "c0_box_drop (BASELINE configs[0], polygon-terrain variant)",
    "c1": "c1_rig (BASELINE configs[1], polygon-terrain variant)",
    "c2": "c2_stress (BASELINE configs[2])",
    "c3": "c3_toi (BASELINE configs[3], 0.02 m boxes for the zero-thickness edges)",
    "c4": "c4_scale (BASELINE configs[4], polygon-terrain variant)",
    "c0e": "c0_box_drop_chain (BASELINE configs[0], its chain terrain; edge shapes, parity unpinned)",
    "c1e": "c1_rig_chain (BASELINE configs[1], its 2000-segment chain; edge shapes, parity unpinned)",
    "c3e": "c3_toi_edges (BASELINE configs[3], zero-thickness edge targets; parity unpinned)",
    "c4e": "c4_scale_chain (BASELINE configs[4], chain terrain; parity unpinned)",
}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def workload_config(args, sc, model, n_bodies, n, world_size):
    """The `config` object of both arms' lines: the workload BASELINE.json names, n worlds per GPU (the reference
    arm times a bounded sample of it, described in its cpu_baseline.sample)."""
    from goib2d import configs
    resets = args.config.startswith("c4")
    return {"workload": WORKLOADS.get(args.config, sc.name),
            "reset_on_fall": "pot below y = -5 -> the world's seeded initial state" if resets else None,
            "worlds_per_gpu": n, "global_worlds": n * world_size, "dt": float(configs.DT),
            "iterations": "8/3", "continuous_physics": True, "contact_capacity": sc.capacity,
            "bodies": int(n_bodies), "fixtures": int(model.fixture_body.shape[0]),
            "candidate_pairs": int(model.pair_a.shape[0]), "parallelism": f"worlds sharded x{world_size}",
            "physics_steps_per_call": args.substeps, "untimed_steps_first": args.skip,
            "l2": "flushed between timed calls (256 MiB write), per-call CUDA events summed"}


# The bounded CPU sample, the same in both arms: the workload's first worlds (CPU_SAMPLE_WORLDS, fewer for c2's
# 256-body worlds), stepped until CPU_SAMPLE_SECONDS have passed or CPU_SAMPLE_MAX_STEPS steps are done.
CPU_SAMPLE_WORLDS = {"c2": 128}
CPU_SAMPLE_SECONDS, CPU_SAMPLE_MAX_STEPS = 10.0, 200


def cpu_sample_worlds(args, n):
    want = args.cpu_sample_worlds or CPU_SAMPLE_WORLDS.get(args.config[:2], 1024)
    return max(1, min(want, n))


def cpu_baseline(sc, model, host, n_sample, threads=0, warmup=True):
    """The parity oracle on the host cores over a bounded sample: the first n_sample worlds, stepped (each step with
    its own actions) until CPU_SAMPLE_SECONDS have passed or CPU_SAMPLE_MAX_STEPS steps are done. Both arms call
    this with the same sample, so their CPU figures are the same measurement."""
    import oracle_lib
    from goib2d import configs
    from goib2d.world import map_state
    sample = map_state(lambda x: np.ascontiguousarray(np.asarray(x)[:n_sample]), host)
    lib = oracle_lib.load(build=False)
    threads = threads or lib.oracle_max_threads()
    na = len(sc.action_joints)
    acts = actions_for(n_sample, CPU_SAMPLE_MAX_STEPS, 0) if na else None  # the workloads with action channels
    if warmup:  # one untimed step of a copy (thread pool start-up, first touches)
        warm = map_state(lambda x: np.array(x, copy=True), sample)
        oracle_lib.step(model, warm, sc.settings, configs.DT, 1, threads=threads, actions=acts[0] if na else None,
                        action_joints=sc.action_joints, action_scale=sc.action_scale)
    t0 = time.perf_counter()
    st, steps = sample, 0
    while steps < CPU_SAMPLE_MAX_STEPS and (steps < 2 or time.perf_counter() - t0 < CPU_SAMPLE_SECONDS):
        st = oracle_lib.step(model, st, sc.settings, configs.DT, 1, threads=threads,
                             actions=acts[steps] if na else None, action_joints=sc.action_joints,
                             action_scale=sc.action_scale)
        steps += 1
    dt = time.perf_counter() - t0
    return {"value": n_sample * steps / dt, "unit": UNIT, "cores": int(threads), "kind": "port", "steps": steps,
            "seconds": dt, "sample": f"{n_sample} worlds x {steps} steps of {sc.name} (the first worlds of the "
                                     f"workload; stepped for {CPU_SAMPLE_SECONDS:.0f} s or {CPU_SAMPLE_MAX_STEPS} steps)"}


def run_reference(args, rank):
    """--impl reference: rank 0 times the oracle (the reference's algorithm, C++) on the host cores. This process
    loads no CUDA library of this repository: the batch's candidate list is built by the host scan."""
    if rank != 0:
        return
    import oracle_lib
    from goib2d import configs
    n = cpu_sample_worlds(args, args.worlds or configs.DEFAULT_N[args.config])
    sc, model, host = configs.batch(args.config, n, args.seed, device_pairs=False)
    oracle_lib.load(build=not (ROOT / "oracle" / "liboracle_goib2d.so").exists())
    cb = cpu_baseline(sc, model, host, n)
    v = cb["value"]
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": cb["steps"],
            "warmup": args.warmup, "ms_per_step": 1000.0 * n / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, goib2d/configs.py)", "impl": "reference",
            "config": workload_config(args, sc, model, host.bodies.type.shape[1],
                                      args.worlds or configs.DEFAULT_N[args.config], args.gpus),
            "cpu_baseline": cb, "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's JAX engine is not installed here; its algorithm runs as the bit-identical C++ "
                    "parity oracle (oracle/), all host threads"}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    import torch
    import torch.distributed as dist
    from goib2d import api, configs, native, shard
    from goib2d.world import map_state
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world_size > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    n = args.worlds or configs.DEFAULT_N[args.config]
    first, _ = shard.world_range(n, rank)  # weak scaling: every rank steps its own n seeded worlds
    # the batch built on the GPU (goib2d_spawn from the host builder's first world and the scene's per-world poses):
    # the same State as configs.batch, without the per-world host builder loop (minutes for c4's 65536 worlds)
    sc, model, state, _, _ = configs.spawn_batch(args.config, n, args.seed, first=first)
    n_cpu = cpu_sample_worlds(args, n)
    host = api.to_host(map_state(lambda t: t[:n_cpu].contiguous(), state))  # the CPU baseline's sample
    eng = api.Engine(model, state.bodies.type.shape[1], sc.action_joints, sc.action_scale)
    K, Wm = args.steps, args.warmup
    na = len(sc.action_joints)
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    # BASELINE c4: every world resets to its seeded initial state when the pot (body 1) falls below y = -5
    resets = args.config.startswith("c4")
    init_state = map_state(torch.clone, state) if resets else None
    reset_count = torch.zeros(n, dtype=torch.int32, device=dev) if resets else None

    S = args.substeps
    acts = torch.from_numpy(actions_for(n, (K + Wm) * S, args.seed, first).reshape(K + Wm, S, n, na)).to(dev) \
        if na else None

    def world_step(a):  # one call: S physics steps of every world (one launch), then the resets (c4)
        eng.step_(state, sc.settings, configs.DT, S, a)
        if resets:
            eng.reset_below(state, init_state, 1, -5.0, reset_count)

    for k0 in range(0, args.skip, S):  # the episode's start, untimed, in calls of S steps like the timed ones
        k1 = min(args.skip, k0 + S)
        skip_acts = torch.from_numpy(actions_for(n, k1 - k0, args.seed + 1000 + k0, first)).to(dev) if na else None
        eng.step_(state, sc.settings, configs.DT, k1 - k0, skip_acts)
        if resets:
            eng.reset_below(state, init_state, 1, -5.0, reset_count)
    for k in range(Wm):
        world_step(acts[k] if na else None)
    torch.cuda.synchronize(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    clocks = Clocks(local_rank)
    if world_size > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    wall0 = time.perf_counter()
    for k in range(K):
        flush.fill_(float(k))
        starts[k].record(stream)
        world_step(acts[Wm + k] if na else None)
        ends[k].record(stream)
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - wall0
    if world_size > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = float(sum(s.elapsed_time(e) for s, e in zip(starts, ends)))
    status = eng.status()
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world_size > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world_size * n * K * S / (ms_max / 1e3)

    # e2e through the public API with host buffers: per call, its S rows of actions read from pinned host memory by
    # the step kernel (mapped memory: the host->device transfer, no separate copy), the S steps, and the pot's
    # observation (position, angle, velocities) written by goib2d_observe into pinned host memory; the host
    # synchronises at the end of the timed region before reading it
    Ke = max(3, min(K, 20))
    a_pin = torch.from_numpy(actions_for(n, Ke * S, args.seed + 1, first).reshape(Ke, S, n, na)).pin_memory() \
        if na else None
    obs_pin = torch.empty((n, 1, 6), dtype=torch.float32).pin_memory()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world_size > 1:
        dist.barrier()
    e0.record(stream)
    for k in range(Ke):
        world_step(a_pin[k] if na else None)
        eng.observe(state, [1], out=obs_pin)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world_size > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world_size * n * Ke * S / (float(te.item()) / 1e3)

    # episode statistics gathered over NCCL (off the timed path): body 1's position / velocity and the status word
    stats = shard.gather_stats(shard.episode_stats(state, 1, status))
    nonfinite = int(((stats[:, 4].to(torch.int32) & 2) != 0).sum().item())

    if rank == 0:
        bytes_ws = state_bytes(state) + (8 if na else 0)
        peak, peak_kind = measured_peak()
        achieved = bytes_ws * n * S / (ms_max / 1e3 / K) / 1e9
        traffic = None
        tp = ROOT / "profiles" / f"traffic_{args.config}.json"
        if tp.exists():
            td = json.loads(tp.read_text())
            traffic = td.get("dram_bytes_per_world_step", 0) * n * S  # per launch group of one call
        cpu = None
        if not args.no_cpu_baseline:
            cpu = cpu_baseline(sc, model, host, n_cpu)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world_size, "steps": K, "warmup": Wm,
            "ms_per_step": ms_max / K, "physics_steps_per_step": S, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded worlds, goib2d/configs.py)",
            "config": workload_config(args, sc, model, host.bodies.type.shape[1], n, world_size),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                         "algorithmic_bytes_per_world_step": bytes_ws,
                         "kernel": (f"one call's launch group ({eng.launches(n, S)} launch(es) for {S} physics "
                                    f"step(s){' + the reset kernel' if resets else ''}), timed as one unit by the "
                                    "per-call CUDA events"),
                         "traffic_source": f"profiles/traffic_{args.config}.json (ncu dram bytes of the launch group)"
                                           if traffic is not None else None},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": n * na * 4 * S * world_size,
                    "d2h_bytes_per_step": n * 6 * 4 * world_size, "steps": Ke,
                    "path": "actions read from pinned host memory by the step kernel; goib2d_observe writes the pot's "
                            "pose and velocity to pinned host memory"},
            "gpu_launches": K * (eng.launches(n, S) + int(resets)), "clocks": clk,
            "wall_s_timed": wall,
            "nonfinite_worlds": nonfinite,
            "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    eng.close()
    if world_size > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
