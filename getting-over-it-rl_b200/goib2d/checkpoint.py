"""Checkpoint and resume of a batched State: its 71 leaves saved to and loaded from one `.npz` file.

The reference engine has no checkpointing of its own: its State is a pure pytree that the caller saves
(goi_jax/box2d/world.py:144-155). Here a State, on the host (numpy) or on the device (torch), is written leaf by leaf
under the leaves' names with a format tag; loading checks that every leaf is present with the dtype and per-world
shape the C ABI gives for the file's bodies, fixture rows, joints and contact slots, and that all leaves hold the
same number of worlds. Stepping a loaded State continues bit for bit where the saved one stopped: the State is the
whole mutable step state (the Model and Settings are the caller's).
"""
import numpy as np

from . import native
from .world import leaf_names, state_from_leaves, state_leaves

FORMAT = "goib2d-state-v1"


def _host(x):
    if hasattr(x, "detach"):  # a torch tensor (device or host)
        return x.detach().cpu().numpy()
    return np.asarray(x)


def save_state(path, state, **meta):
    """Write `state` (batched: every leaf (N, ...)) to `path` (.npz). meta: extra scalars or strings stored beside the
    leaves (e.g. the episode step), returned by load_state."""
    leaves = [_host(x) for x in state_leaves(state)]
    n = leaves[0].shape[0] if leaves[0].ndim else None
    if n is None or any(x.ndim == 0 or x.shape[0] != n for x in leaves):
        raise ValueError("save_state needs a batched State (every leaf with the same leading world axis)")
    arrays = {name: np.ascontiguousarray(x) for name, x in zip(leaf_names(), leaves)}
    for k, v in meta.items():
        if k in arrays or k.startswith("__"):
            raise ValueError(f"meta key {k!r} is reserved")
        arrays["meta." + k] = np.asarray(v)
    np.savez(path, __format__=np.asarray(FORMAT), **arrays)


def load_state(path, device=None):
    """(State, meta) from a save_state file: numpy leaves, or torch tensors on `device` (e.g. "cuda") when given."""
    with np.load(path, allow_pickle=False) as f:
        if "__format__" not in f.files or str(f["__format__"]) != FORMAT:
            raise ValueError(f"{path}: not a {FORMAT} file")
        names = leaf_names()
        missing = [k for k in names if k not in f.files]
        if missing:
            raise ValueError(f"{path}: missing leaves {missing[:4]}{'...' if len(missing) > 4 else ''}")
        leaves = [f[k] for k in names]
        meta = {k[5:]: f[k][()] for k in f.files if k.startswith("meta.")}
    n = leaves[0].shape[0]
    B = leaves[names.index("bodies.type")].shape[1]
    rows = leaves[names.index("fixtures.friction")].shape[1]
    J = leaves[names.index("joints.motor_speed")].shape[1]
    C = leaves[names.index("contacts.pair")].shape[1]
    for (name, shape, dt), x in zip(native.leaf_spec(B, rows, J, C), leaves):
        if x.shape != (n,) + tuple(shape) or x.dtype != dt:
            raise ValueError(f"{path}: leaf {name} is {x.dtype}{x.shape}, expected {dt}{(n,) + tuple(shape)}")
    state = state_from_leaves(leaves)
    if device is not None:
        from . import api
        state = api.to_device(state, device)
    return state, meta
