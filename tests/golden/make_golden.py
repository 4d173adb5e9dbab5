"""Generate the golden vectors: the reference engine's own states, stepped by the reference's own Python code.

    python tests/golden/make_golden.py --reference PATH [--jobs 8] [--only NAME ...]

PATH is a checkout of miwate/getting-over-it-rl (or the GOIB2D_REFERENCE environment variable); it is read, never
written, and only this generator needs it.

The reference (goi_jax/box2d) is JAX; jax is not installed here, so `tests/golden/jaxshim` stands in for it with
numpy (one world at a time, JAX's float32/int32 dtype rules, `.at[]` updates, eager control flow). The reference's
scene builders run unchanged: its tests' scenes (tests/box2d/box2d_scenes.py, tests/box2d/test_toi.py) through a
recording stand-in for their `Twin` harness, and this repo's benchmark workloads (goib2d/configs.py) through the
reference's WorldDef. Each scene is written to tests/golden/<name>.npz:

    meta                JSON: scene name, Settings, contact capacity, dt, checkpoint steps, builder-call log
    model.<field>       the reference's Model after build (compact layout for the workloads)
    traj.<leaf>         the reference's State leaf after each checkpoint step, stacked on a new first axis
                        (checkpoint 0 is the built state); leaves as in goib2d.world.leaf_names()

The builder-call log lets tests replay the same calls through goib2d.WorldDef and compare with the model and the
built state.
"""
import argparse
import json
import multiprocessing as mp
import os
import sys
import time
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REFERENCE = Path(os.environ.get("GOIB2D_REFERENCE", "reference"))

GAME_SCENES = ["free_fall", "box_on_ground", "box_stack", "polygons_at_angles", "polygon_circle", "revolute",
               "prismatic", "weld", "pile", "misc", "late_wake", "thin_plates", "limits_mid_run"]
TOI_SCENES = ["ball_wall", "poly_angles", "hammer_chain", "multi_event", "stock_bullets", "island_walk"]
STOCK_SCENES = ["box_stack", "pile", "revolute", "prismatic", "weld", "polygon_circle", "misc"]
CONFIG_JOBS = [("c0", 0, 60), ("c1", 0, 60), ("c1", 1, 60), ("c2", 0, 12), ("c3", 0, 30), ("c4", 0, 30)]


def checkpoints(steps):
    ks = [1, 2, 3, 5, 10, 20, 30, 45, 60, 90, 120, 180, 240]
    return [k for k in ks if k <= steps] + ([steps] if steps not in ks else [])


def _jsonable(x):
    if isinstance(x, np.ndarray):
        return [_jsonable(v) for v in x.tolist()]
    if isinstance(x, (list, tuple)):
        return [_jsonable(v) for v in x]
    if isinstance(x, dict):
        return {k: _jsonable(v) for k, v in x.items()}
    if isinstance(x, (np.floating, float)):
        return float(x)
    if isinstance(x, (np.integer,)):
        return int(x)
    if isinstance(x, (np.bool_,)):
        return bool(x)
    return x


def setup_reference():
    """Import the reference engine with the numpy stand-in for jax, and stub the modules its scene files import
    that need the (unbuilt) Box2D oracle library."""
    REFERENCE = Path(os.environ.get("GOIB2D_REFERENCE", "reference"))
    sys.path.insert(0, str(HERE / "jaxshim"))
    sys.path.insert(0, str(REFERENCE))
    sys.path.insert(0, str(REFERENCE / "tests" / "box2d"))
    sys.path.insert(0, str(REPO / "getting-over-it-rl_b200"))
    from goi_jax import box2d as jb
    ref = types.ModuleType("goi_jax.reference")
    rb = types.ModuleType("goi_jax.reference.box2d")
    rb.deg2rad = jb.settings.deg2rad
    rs = types.ModuleType("goi_jax.reference.scene")
    rs.DEFAULT_DUMP = Path("/nonexistent/engine-dump-start.jsonl")
    ref.box2d, ref.scene = rb, rs
    sys.modules.update({"goi_jax.reference": ref, "goi_jax.reference.box2d": rb, "goi_jax.reference.scene": rs})

    class Recorder:
        """The reference WorldDef with every add_* call logged."""
        default_settings = None

        def __init__(self, settings=None, layer_masks=None, contact_capacity=16, **_oracle_kw):
            self.settings = settings or Recorder.default_settings or jb.Settings.game()
            self.layer_masks = layer_masks
            self.defn = jb.WorldDef(self.settings, layer_masks=layer_masks)
            self.capacity = contact_capacity
            self.calls = []

        def __getattr__(self, name):
            if not name.startswith("add_"):
                raise AttributeError(name)

            def call(*a, **k):
                self.calls.append([name, _jsonable(list(a)), _jsonable(k)])
                return getattr(self.defn, name)(*a, **k)
            return call

    harness = types.ModuleType("box2d_harness")
    harness.Twin, harness.H = Recorder, jb.GAME_DT
    harness.QUANTITIES = ()
    harness.compare = harness.jax_snapshot = harness.ref_snapshot = None
    sys.modules["box2d_harness"] = harness
    return jb, Recorder


def leaves_of(state, names):
    from goib2d.world import state_leaves
    return dict(zip(names, [np.asarray(x) for x in state_leaves(state)]))


def run_job(job):
    kind, name, arg = job
    t0 = time.time()
    jb, Recorder = setup_reference()
    from goib2d import configs
    from goib2d.world import leaf_names
    names = leaf_names()
    if kind in ("game", "stock", "toi"):
        if kind == "toi":
            import test_toi as scenes
        else:
            import box2d_scenes as scenes
        # The scene module binds the harness's Twin when it is first imported. Each job runs in a fresh interpreter
        # (maxtasksperchild=1), so that Twin is this job's Recorder; the assertion keeps a reused worker from
        # handing one job's default settings to the next.
        assert scenes.Twin is Recorder, "scene module bound another job's recorder"
        maker = scenes.SCENES[name]
        Recorder.default_settings = jb.Settings.stock() if kind == "stock" else None
        rec = maker()
        expect = jb.Settings.stock() if kind == "stock" else jb.Settings.game()
        if kind != "toi":  # the TOI scenes pass their own settings (continuous physics, the pair rule)
            assert _settings_dict(rec.settings) == _settings_dict(expect), f"{kind}_{name}: settings differ"
        settings, cap, dt = rec.settings, rec.capacity, jb.GAME_DT
        model, state = rec.defn.build(cap)
        steps = {"game": 240 if name == "late_wake" else 60, "stock": 60, "toi": 40}[kind]
        meta = dict(name=f"{kind}_{name}", source=kind, scene=name, capacity=cap, dt=float(dt),
                    settings=_settings_dict(settings), layer_masks=_jsonable(rec.layer_masks), calls=rec.calls,
                    compact=False)
    else:
        world, steps = arg
        sc = configs.scene(name, 0, n=4)
        rec = Recorder(sc.settings, contact_capacity=sc.capacity)
        sc.build_world(rec, world)
        settings, cap, dt = sc.settings, sc.capacity, configs.DT
        model, state = rec.defn.build(cap)
        from goi_jax.box2d import world as W
        model = W.compact_model(model, state)
        state = W.compact_state(model, state)
        meta = dict(name=f"{name}_w{world}", source="config", scene=name, seed=0, world=world, capacity=cap,
                    dt=float(dt), settings=_settings_dict(settings), layer_masks=None, calls=rec.calls, compact=True)
    ks = checkpoints(steps)
    meta["checkpoints"] = [0] + ks
    out = {"meta": np.array(json.dumps(meta))}
    for f in model._fields:
        v = getattr(model, f)
        if v is not None:
            out[f"model.{f}"] = np.asarray(v)
    traj = {leaf: [v] for leaf, v in leaves_of(state, names).items()}
    st = state
    for k in range(1, steps + 1):
        st = jb.step(model, st, settings, dt)
        if k in ks:
            for leaf, v in leaves_of(st, names).items():
                traj[leaf].append(v)
    for leaf, vs in traj.items():
        out[f"traj.{leaf}"] = np.stack(vs, 0)
    path = HERE / f"{meta['name']}.npz"
    np.savez_compressed(path, **out)
    return f"{meta['name']}: {steps} steps, {time.time() - t0:.0f} s"


def _settings_dict(s):
    from dataclasses import fields
    d = {}
    for f in fields(s):
        v = getattr(s, f.name)
        d[f.name] = [float(x) for x in v] if isinstance(v, tuple) else (
            float(v) if isinstance(v, (float, np.floating)) else v)
    return d


def all_jobs():
    jobs = [("game", n, None) for n in GAME_SCENES] + [("toi", n, None) for n in TOI_SCENES]
    jobs += [("stock", n, None) for n in STOCK_SCENES]
    jobs += [("config", n, (w, steps)) for n, w, steps in CONFIG_JOBS]
    return jobs


def job_name(job):
    kind, name, arg = job
    return f"{name}_w{arg[0]}" if kind == "config" else f"{kind}_{name}"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--only", nargs="*")
    ap.add_argument("--reference", default=None, help="checkout of the reference repository")
    args = ap.parse_args()
    if args.reference:
        os.environ["GOIB2D_REFERENCE"] = str(Path(args.reference).resolve())
    jobs = all_jobs()
    if args.only:
        jobs = [j for j in jobs if job_name(j) in args.only]
    # slowest first
    weight = {"late_wake": 9, "pile": 8, "c2": 7, "c3": 6, "c4": 6, "island_walk": 5, "multi_event": 5}
    jobs.sort(key=lambda j: -weight.get(j[1], 1))
    with mp.get_context("spawn").Pool(args.jobs, maxtasksperchild=1) as pool:
        for msg in pool.imap_unordered(run_job, jobs):
            print(msg, flush=True)


if __name__ == "__main__":
    main()
