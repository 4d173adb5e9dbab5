"""A numpy stand-in for the slice of `jax` that the reference engine (goi_jax/box2d, XLA path) uses.

Test infrastructure only: `tests/golden/make_golden.py` puts this package first on sys.path so that the reference's
own Python engine can be imported and stepped in a container without jax, to record golden vectors. It runs ONE
world at a time (no vmap); arrays are numpy arrays with JAX's x64-disabled dtype rules (float32 / int32 defaults,
float64 inputs canonicalised to float32) and JAX's `.at[...]` update syntax.
"""
from types import SimpleNamespace

from . import lax, numpy  # noqa: F401
from .numpy import Arr, _tree_leaves, _tree_map


class _Tracer:  # nothing here is ever traced
    pass


core = SimpleNamespace(Tracer=_Tracer)


class TracerArrayConversionError(Exception):
    pass


errors = SimpleNamespace(TracerArrayConversionError=TracerArrayConversionError)
tree = SimpleNamespace(map=_tree_map, leaves=_tree_leaves)
tree_util = SimpleNamespace(tree_map=_tree_map, tree_leaves=_tree_leaves)


def jit(f=None, **_kw):
    if f is None:
        return lambda g: g
    return f


def block_until_ready(x):
    return x


def vmap(*_a, **_k):
    raise NotImplementedError("the numpy stand-in runs one world at a time")


__all__ = ["Arr", "core", "errors", "jit", "lax", "numpy", "tree", "block_until_ready"]
