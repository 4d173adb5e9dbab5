"""`jax.lax` control flow and bit casts for one (unbatched) world, eagerly in Python."""
import numpy as _np

from .numpy import _plain, _wrap


def while_loop(cond, body, init):
    c = init
    while bool(cond(c)):
        c = body(c)
    return c


def fori_loop(lo, hi, body, init):
    c = init
    for i in range(int(lo), int(hi)):
        c = body(_np.int32(i), c)
    return c


def switch(index, branches, *operands):
    i = int(_np.clip(int(index), 0, len(branches) - 1))
    return branches[i](*operands)


def cond(pred, true_fn, false_fn, *operands):
    return true_fn(*operands) if bool(pred) else false_fn(*operands)


def pmax(x, axis_name):
    return x


def optimization_barrier(x):
    return x


def bitcast_convert_type(x, dtype):
    a = _np.asarray(_plain(x))
    return _wrap(a.view(_np.dtype(dtype)).copy())
