"""The device-side API: States in HBM (torch tensors as device memory) stepped by libgoib2d.so.

    engine = Engine(model)                       # uploads the Model once (goib2d_model_create)
    dev = to_device(broadcast(state, 4096))      # batched State, leaves (N, ...) on cuda
    step_(model, dev, settings, dt, n_steps=10)  # in place, asynchronous on the current stream
    new = step(model, dev, settings, dt)         # pure, like the reference's step

`step(model, state, settings, dt, axis_name=None)` keeps the reference's signature (goi_jax/box2d/step.py:28): state
in, new state out. `axis_name` is accepted and ignored: the batch is whatever leading axis the leaves carry. The
Model is passed each call, as in the reference; its device copy is cached per (Model object, device).
There is no CPU path: without the library every call raises.
"""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import torch

from . import native
from .settings import Settings, settings_struct
from .world import State, leaf_names, map_state, state_from_leaves, state_leaves

HERE = Path(__file__).resolve().parent
CSRC = HERE.parent / "csrc"

_TORCH = {np.dtype(np.float32): torch.float32, np.dtype(np.int32): torch.int32, np.dtype(np.bool_): torch.bool}


def build(out=None):
    """Compile libgoib2d.so for sm_100a in-tree (csrc/build.sh)."""
    out = Path(out or native.lib_path())
    subprocess.run(["sh", str(CSRC / "build.sh"), str(out)], check=True)
    return out


class Engine:
    """A Model uploaded to the current CUDA device (one goib2d_model handle)."""

    def __init__(self, model, n_bodies=None, action_joints=(), action_scale=()):
        self.lib = native.load()
        if n_bodies is None:
            n_bodies = _n_bodies(model)
        self.n_bodies = int(n_bodies)
        self.model = model
        packed = native.model_desc(model, self.n_bodies)
        h = C.c_void_p()
        native.check(self.lib.goib2d_model_create(C.byref(packed.desc), C.byref(h)))
        self.handle = h
        self.device = torch.cuda.current_device()
        self.n_action = 0
        self._bound = None     # (State, its first leaf's address, checked pointer table): see _bind
        self._settings = None  # (Settings, its C struct)
        if len(action_joints):
            self.set_action_map(action_joints, action_scale)

    def set_action_map(self, joints, scale):
        j = np.ascontiguousarray(joints, np.int32)
        s = np.ascontiguousarray(scale, np.float32)
        native.check(self.lib.goib2d_model_set_action_map(self.handle, len(j), j.ctypes.data_as(native._i),
                                                          s.ctypes.data_as(native._f)))
        self.n_action = len(j)

    def _bind(self, state):
        """The checked leaf pointer table of a device State, cached for the last State object stepped (a State is
        immutable, so the same object has the same leaves; the first leaf's address guards against storage
        changes)."""
        c = self._bound
        if c is not None and c[0] is state and c[1] == state.bodies.type.data_ptr():
            return c[2]
        leaves = state_leaves(state)
        first = leaves[0]
        if not (isinstance(first, torch.Tensor) and first.is_cuda):
            raise TypeError("step_ needs a device State (goib2d.to_device)")
        n = first.shape[0]
        if state.bodies.type.shape[1] != self.n_bodies or state.joints.motor_speed.shape[1] != len(self.model.joint_type):
            raise ValueError(f"State has {state.bodies.type.shape[1]} bodies / {state.joints.motor_speed.shape[1]} joints,"
                             f" the Model {self.n_bodies} / {len(self.model.joint_type)}")
        for t in leaves:
            if not t.is_contiguous() or t.device != first.device:
                raise ValueError("State leaves must be contiguous tensors on one device")
        bound = (n, state.contacts.pair.shape[1], state.fixtures.friction.shape[1], first.device,
                 (C.c_void_p * len(leaves))(*[t.data_ptr() for t in leaves]))
        self._bound = (state, state.bodies.type.data_ptr(), bound)
        return bound

    def step_(self, state, settings, dt, n_steps=1, actions=None, stream=None):
        """Step every world of a batched device State n_steps times, in place; returns the State. actions: None, a
        float32 (N, n_action) tensor used before every step, or (n_steps, N, n_action) with one row per step
        (goib2d_step_seq); on the device or in pinned host memory. All n_steps steps run in one launch where the
        batch takes the one-kernel step (launches())."""
        n, C_, rows, device, ptrs = self._bind(state)
        if self._settings is None or self._settings[0] is not settings:
            self._settings = (settings, settings_struct(settings))
        ss = self._settings[1]
        act, stride = None, 0
        if actions is not None:
            if not (isinstance(actions, torch.Tensor) and actions.dtype == torch.float32 and
                    (actions.is_cuda or actions.is_pinned())):
                raise TypeError("actions must be a float32 tensor on the device or in pinned host memory")
            per_step = (int(n_steps), n, self.n_action)
            if tuple(actions.shape) == per_step:
                stride = n * self.n_action
            elif tuple(actions.shape) != (n, self.n_action):
                raise ValueError(f"actions must be ({n}, {self.n_action}) or {per_step}")
            if not actions.is_contiguous():
                raise ValueError("actions must be contiguous")
            act = actions.data_ptr()
        if stream is None:
            stream = torch.cuda.current_stream(device).cuda_stream
        native.check(self.lib.goib2d_step_seq(self.handle, C.addressof(ss), C.c_float(float(dt)), C_, rows, n,
                                              int(n_steps), ptrs, act, stride, stream))
        return state

    def launches(self, n_worlds, n_steps):
        """Kernel launches one step_ call of n_steps steps over n_worlds worlds makes (goib2d_launches)."""
        k = self.lib.goib2d_launches(self.handle, int(n_worlds), int(n_steps))
        native.check(min(k, 0))
        return k

    # ---- env helpers (goib2d_reset_*, goib2d_observe, goib2d_raycast): device tensors in and out, on the State's
    # current stream; no counterpart in the reference engine.

    def _stream(self, device):
        return torch.cuda.current_stream(device).cuda_stream

    def reset_masked(self, state, init_state, mask):
        """Worlds with mask[w] set (bool/uint8 cuda tensor (N,)) get every leaf's row from init_state (a device
        State of the same shape: each world's initial state)."""
        n, C_, rows, device, ptrs = self._bind(state)
        init = (C.c_void_p * len(ptrs))(*[t.data_ptr() for t in state_leaves(init_state)])
        m = mask.to(torch.uint8).contiguous()
        native.check(self.lib.goib2d_reset_masked(self.handle, C_, rows, n, ptrs, init, m.data_ptr(),
                                                  self._stream(device)))
        return state

    def reset_below(self, state, init_state, body, y_min, counts=None):
        """BASELINE c4's reset-on-fall: the worlds whose `body` has c.y < y_min are reset to init_state; counts
        (int32 cuda tensor (N,), optional) counts the resets per world."""
        n, C_, rows, device, ptrs = self._bind(state)
        init = (C.c_void_p * len(ptrs))(*[t.data_ptr() for t in state_leaves(init_state)])
        cp = counts.data_ptr() if counts is not None else None
        native.check(self.lib.goib2d_reset_below(self.handle, C_, rows, n, ptrs, init, int(body), C.c_float(y_min),
                                                 cp, self._stream(device)))
        return state

    def observe(self, state, bodies, out=None):
        """(N, len(bodies), 6) float32: c.x, c.y, angle, v.x, v.y, w of the given bodies. out may be a pinned host
        tensor: the kernel writes it directly (synchronise the stream before reading it)."""
        n, C_, rows, device, ptrs = self._bind(state)
        b = np.ascontiguousarray(bodies, np.int32)
        if out is None:
            out = torch.empty((n, len(b), 6), dtype=torch.float32, device=device)
        native.check(self.lib.goib2d_observe(self.handle, C_, rows, n, ptrs, len(b), b.ctypes.data_as(native._i),
                                             out.data_ptr(), self._stream(device)))
        return out

    def raycast(self, state, body, n_rays, max_length, out=None):
        """(N, n_rays) float32: nearest hit fraction of ray k from `body`'s centre of mass at angle 2 pi k / n_rays
        over the static level (1 = no hit within max_length)."""
        n, C_, rows, device, ptrs = self._bind(state)
        if out is None:
            out = torch.empty((n, n_rays), dtype=torch.float32, device=device)
        native.check(self.lib.goib2d_raycast(self.handle, C_, rows, n, ptrs, int(body), int(n_rays),
                                             C.c_float(max_length), out.data_ptr(), self._stream(device)))
        return out

    def spawn(self, template, n_worlds, first_body, placements, speed_joints=(), speeds=None):
        """A new device State of n_worlds worlds built on the device (goib2d_spawn): each a copy of `template` (a
        one-world device State, e.g. world 0's build) with bodies first_body .. first_body + k - 1 placed as the
        builder's add_body places them, from placements (float32 (n_worlds, k, 6): x, y, angle, v.x, v.y, w; device
        or pinned host), and joint speed_joints[j]'s motor speed = speeds[:, j] (float32 (n_worlds, len)). The
        result equals building every world through WorldDef with those poses."""
        leaves = state_leaves(template)
        first = leaves[0]
        if not (isinstance(first, torch.Tensor) and first.is_cuda and first.shape[0] == 1):
            raise TypeError("spawn needs a one-world device State as its template")
        out = state_from_leaves([torch.empty((n_worlds,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
                                 for t in leaves])
        n, C_, rows, device, ptrs = self._bind(out)
        tmpl = (C.c_void_p * len(leaves))(*[t.data_ptr() for t in leaves])
        pl = placements.to(device=device, dtype=torch.float32).contiguous()
        if pl.dim() != 3 or pl.shape[0] != n_worlds or pl.shape[2] != 6:
            raise ValueError(f"placements must be (n_worlds, k, 6), got {tuple(pl.shape)}")
        sj = np.ascontiguousarray(speed_joints, np.int32)
        sp = None
        if len(sj):
            sp = speeds.to(device=device, dtype=torch.float32).reshape(n_worlds, len(sj)).contiguous()
        native.check(self.lib.goib2d_spawn(self.handle, C_, rows, n, ptrs, tmpl, int(first_body), int(pl.shape[1]),
                                           pl.data_ptr(), len(sj), sj.ctypes.data_as(native._i),
                                           sp.data_ptr() if sp is not None else None, self._stream(device)))
        return out

    def kernels_per_step(self, n_worlds):
        """Kernel launches one step of n_worlds worlds of this model makes (goib2d_kernels_per_step)."""
        k = self.lib.goib2d_kernels_per_step(self.handle, int(n_worlds))
        native.check(min(k, 0))
        return k

    def set_step_mode(self, mode):
        """Worlds per warp of the one-launch step (batches below 16384 worlds): 0 chosen per batch, 1 or 2. Results
        are identical in every mode."""
        native.check(self.lib.goib2d_set_step_mode(self.handle, int(mode)))

    def set_state_staging(self, max_bytes_per_world):
        """Keep up to this many bytes of each world's State rows in shared memory across a one-launch call (0, the
        default: none). Results are identical either way."""
        native.check(self.lib.goib2d_set_state_staging(self.handle, int(max_bytes_per_world)))

    def set_checks(self, on=True):
        """Checked stepping: each later step validates the State's index fields first and raises (stepping nothing)
        when a world's are out of range (goib2d_set_checks)."""
        native.check(self.lib.goib2d_set_checks(self.handle, int(bool(on))))

    def validate(self, state):
        """(first bad world, its leaf name) of a device State, or None when every index field is in range
        (goib2d_validate; synchronises)."""
        n, C_, rows, device, ptrs = self._bind(state)
        bw, bl = C.c_int64(-1), C.c_int32(-1)
        native.check(self.lib.goib2d_validate(self.handle, C_, rows, n, ptrs, C.byref(bw), C.byref(bl),
                                              self._stream(device)))
        return None if bw.value < 0 else (bw.value, leaf_names()[bl.value])

    def set_event_log(self, capacity):
        """Log each world's contact events (Begin / End / PostSolve, goib2d_event) of every step, capacity per world
        (0: off)."""
        native.check(self.lib.goib2d_set_event_log(self.handle, int(capacity)))

    def events(self):
        """The last step's event log: (events (n_worlds, capacity) of native.EVENT_DTYPE, counts (n_worlds,))
        copied to the host; a count above capacity means the later events were dropped."""
        ev, cnt, n, cap = C.c_void_p(), C.c_void_p(), C.c_int64(), C.c_int32()
        native.check(self.lib.goib2d_events(self.handle, C.byref(ev), C.byref(cnt), C.byref(n), C.byref(cap)))
        N, K = n.value, cap.value
        out = np.zeros((N, K), native.EVENT_DTYPE)
        counts = np.zeros(N, np.int32)
        if N and K:
            native.check(self.lib.goib2d_events_copy(self.handle, out.ctypes.data, counts.ctypes.data_as(native._i), N))
        return out, counts

    def status(self):
        """Per-world status words of the last step, copied to the host (numpy int32; see goib2d_status)."""
        n = C.c_int64()
        p = C.c_void_p()
        native.check(self.lib.goib2d_status(self.handle, C.byref(p), C.byref(n)))
        out = np.zeros(n.value, np.int32)
        if n.value:
            native.check(self.lib.goib2d_status_copy(self.handle, out.ctypes.data_as(native._i), n.value))
        return out

    def close(self):
        if getattr(self, "handle", None):
            self.lib.goib2d_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _n_bodies(model):
    fb = np.asarray(model.fixture_body)
    ja, jb = np.asarray(model.joint_a), np.asarray(model.joint_b)
    tb = model.toi_bodies
    if tb is not None:
        return int(np.asarray(tb).shape[0])
    return int(max([fb.max(initial=-1), ja.max(initial=-1), jb.max(initial=-1)]) + 1)


_ENGINES = {}


def engine_for(model, n_bodies=None):
    key = (id(model), torch.cuda.current_device())
    e = _ENGINES.get(key)
    if e is None:
        if len(_ENGINES) >= 32:
            _ENGINES.pop(next(iter(_ENGINES))).close()
        e = Engine(model, n_bodies)
        _ENGINES[key] = e
    return e


def broadcast(state, n):
    """n copies of a single-world numpy State, as a batched numpy State."""
    return map_state(lambda x: np.ascontiguousarray(np.broadcast_to(np.asarray(x), (n,) + np.shape(x))), state)


def to_device(state, device="cuda"):
    """A numpy State (batched) as torch tensors on the device."""
    return map_state(lambda x: torch.from_numpy(np.array(x, copy=True, order="C")).to(device), state)


def to_host(state):
    return map_state(lambda x: x.cpu().numpy() if isinstance(x, torch.Tensor) else np.asarray(x), state)


def step_(model, state, settings, dt, n_steps=1, actions=None, stream=None):
    """In-place batched step of a device State (leaves (N, ...) torch cuda tensors)."""
    B = state.bodies.type.shape[1]
    return engine_for(model, B).step_(state, settings, dt, n_steps, actions, stream)


def step(model, state, settings, dt, axis_name=None):
    """b2World::Step of every world of `state` (device tensors, leading world axis; a single-world State gets one
    and loses it again). Pure: returns a new State."""
    leaves = state_leaves(state)
    single = leaves[0].dim() == 1
    out = state_from_leaves([(t.unsqueeze(0) if single else t).clone().contiguous() for t in leaves])
    step_(model, out, settings, dt)
    if single:
        out = state_from_leaves([t[0] for t in state_leaves(out)])
    return out


__all__ = ["Engine", "build", "step", "step_", "to_device", "to_host", "broadcast", "State", "Settings"]


def seed_placements(rule, seed, first_world, n_worlds, device="cuda"):
    """goib2d_seed_placements: (placements (n_worlds, k, 6), speeds (n_worlds,) or None) drawn on the device for
    worlds first_world .. first_world + n_worlds - 1 of a scene seeded `seed` (rule: native.SpawnRule; its heights
    and discs must be device or pinned host memory kept alive by the caller)."""
    lib = native.load()
    k = 3 if rule.kind == native.SPAWN_RIG else int(rule.n_bodies)
    pl = torch.empty((n_worlds, k, 6), dtype=torch.float32, device=device)
    sp = torch.empty(n_worlds, dtype=torch.float32, device=device) if rule.kind == native.SPAWN_RIG else None
    stream = torch.cuda.current_stream(pl.device).cuda_stream
    native.check(lib.goib2d_seed_placements(C.byref(rule), C.c_uint64(seed & (2**64 - 1)), int(first_world),
                                            int(n_worlds), pl.data_ptr(), sp.data_ptr() if sp is not None else None,
                                            stream))
    return pl, sp
