"""`jax.numpy` on numpy, x64 disabled: float64 -> float32, int64 -> int32, uint64 -> uint32 wherever a value enters
or leaves an operation; Python scalars stay weakly typed (numpy 2 / NEP 50 gives the same promotion as JAX for
them). Arrays are `Arr`, an ndarray subclass that adds JAX's functional `.at[idx].set/min/max/add(..., mode=)`."""
import builtins as _b

import numpy as _np

float32, int32, uint32, bool_ = _np.float32, _np.int32, _np.uint32, _np.bool_
ndarray = _np.ndarray
inf = _np.inf
iinfo = _np.iinfo
finfo = _np.finfo

_CANON = {_np.dtype(_np.float64): _np.dtype(_np.float32), _np.dtype(_np.int64): _np.dtype(_np.int32),
          _np.dtype(_np.uint64): _np.dtype(_np.uint32)}


def _canon_dtype(dt):
    dt = _np.dtype(dt)
    return _CANON.get(dt, dt)


def _plain(x):
    """Input canonicalisation: numpy arrays/scalars of 64-bit types are cast down; Python scalars left weak."""
    if isinstance(x, Arr):
        return x.view(_np.ndarray)
    if isinstance(x, (_np.ndarray, _np.generic)):
        c = _canon_dtype(x.dtype)
        return x.astype(c) if c != x.dtype else x
    return x


def _wrap(x):
    """Output canonicalisation: arrays become Arr; 64-bit results are cast down; numpy scalars stay scalars."""
    if isinstance(x, _np.ndarray):
        c = _canon_dtype(x.dtype)
        if c != x.dtype:
            x = x.astype(c)
        return x.view(Arr)
    if isinstance(x, _np.generic):
        c = _canon_dtype(x.dtype)
        return x.astype(c) if c != x.dtype else x
    return x


class _AtIndex:
    def __init__(self, arr, idx):
        self.arr, self.idx = arr, idx

    def _apply(self, val, mode, op):
        base = _np.array(self.arr.view(_np.ndarray), copy=True)
        idx = self.idx
        val = _plain(val)
        if isinstance(idx, tuple) or isinstance(idx, slice) or idx is Ellipsis:
            if op == "set":
                base[idx] = val
            else:
                getattr(_np, op).at(base, idx, val)
            return base.view(Arr)
        idx = _np.asarray(_plain(idx))
        n = base.shape[0]
        if idx.ndim == 0:
            i = int(idx)
            if i < 0:
                i += n
            if not 0 <= i < n:
                if mode in ("drop", "fill"):
                    return base.view(Arr)
                i = _b.min(_b.max(i, 0), n - 1)  # JAX clamps out-of-range updates by default
            if op == "set":
                base[i] = val
            else:
                getattr(_np, op).at(base, i, val)
            return base.view(Arr)
        ii = _np.where(idx < 0, idx + n, idx)
        ok = (ii >= 0) & (ii < n)
        vb = _np.broadcast_to(_np.asarray(val, dtype=base.dtype), ii.shape + base.shape[1:])
        if mode in ("drop", "fill"):
            ii, vb = ii[ok], vb[ok]
        else:
            ii = _np.clip(ii, 0, n - 1)
        if op == "set":
            base[ii] = vb
        else:
            getattr(_np, op).at(base, ii, vb)
        return base.view(Arr)

    def set(self, val, mode=None):
        return self._apply(val, mode, "set")

    def min(self, val, mode=None):
        return self._apply(val, mode, "minimum")

    def max(self, val, mode=None):
        return self._apply(val, mode, "maximum")

    def add(self, val, mode=None):
        return self._apply(val, mode, "add")


class _At:
    def __init__(self, arr):
        self.arr = arr

    def __getitem__(self, idx):
        return _AtIndex(self.arr, idx)


class Arr(_np.ndarray):
    @property
    def at(self):
        return _At(self)

    def __array_ufunc__(self, ufunc, method, *inputs, **kwargs):
        ins = tuple(_plain(x) for x in inputs)
        if "out" in kwargs:
            kwargs["out"] = tuple(_plain(o) for o in kwargs["out"])
        res = getattr(ufunc, method)(*ins, **kwargs)
        if isinstance(res, tuple):
            return tuple(_wrap(r) for r in res)
        return _wrap(res)

    def astype(self, dtype, *a, **k):
        return _wrap(self.view(_np.ndarray).astype(dtype, *a, **k))


# ---- constructors


def _default_dtype(v):
    if isinstance(v, bool) or isinstance(v, _np.bool_):
        return _np.bool_
    if isinstance(v, int):
        return _np.int32
    if isinstance(v, float):
        return _np.float32
    return _canon_dtype(_np.asarray(v).dtype)


def asarray(x, dtype=None):
    if dtype is None:
        if isinstance(x, (bool, int, float)):
            dtype = _default_dtype(x)
        else:
            return _wrap(_np.array(_plain(x), copy=True) if isinstance(x, (list, tuple)) else _np.asarray(_plain(x)).copy())
    return _wrap(_np.asarray(_plain(x)).astype(_canon_dtype(dtype)))


array = asarray


def zeros(shape, dtype=_np.float32):
    return _wrap(_np.zeros(shape, _canon_dtype(dtype)))


def ones(shape, dtype=_np.float32):
    return _wrap(_np.ones(shape, _canon_dtype(dtype)))


def full(shape, fill, dtype=None):
    dt = _canon_dtype(dtype) if dtype is not None else _default_dtype(fill)
    return _wrap(_np.full(shape, _plain(fill), dt))


def zeros_like(x, dtype=None):
    return _wrap(_np.zeros(_np.shape(x), _canon_dtype(dtype or _np.asarray(x).dtype)))


def ones_like(x, dtype=None):
    return _wrap(_np.ones(_np.shape(x), _canon_dtype(dtype or _np.asarray(x).dtype)))


def full_like(x, fill, dtype=None):
    return _wrap(_np.full(_np.shape(x), _plain(fill), _canon_dtype(dtype or _np.asarray(x).dtype)))


def arange(*args, dtype=None):
    if dtype is None:
        dtype = _np.float32 if _b.any(isinstance(a, float) for a in args) else _np.int32
    return _wrap(_np.arange(*[int(a) if isinstance(a, (_np.integer,)) else a for a in args], dtype=_canon_dtype(dtype)))


# ---- elementwise / selection


def where(c, x, y):
    return _wrap(_np.where(_plain(c), _plain(x), _plain(y)))


def _u(fn):
    return lambda *a, **k: _wrap(fn(*[_plain(x) for x in a], **k))


sqrt, floor, isnan, minimum, maximum = _u(_np.sqrt), _u(_np.floor), _u(_np.isnan), _u(_np.minimum), _u(_np.maximum)
round = _u(_np.round)  # noqa: A001  (half to even, as jnp.round)
mod = _u(_np.mod)
abs = _u(_np.abs)  # noqa: A001


def clip(x, lo=None, hi=None):
    return _wrap(_np.clip(_plain(x), _plain(lo), _plain(hi)))


def stack(xs, axis=0):
    return _wrap(_np.stack([_np.asarray(_plain(x)) for x in xs], axis))


def concatenate(xs, axis=0):
    return _wrap(_np.concatenate([_np.asarray(_plain(x)) for x in xs], axis))


def broadcast_to(x, shape):
    return _wrap(_np.array(_np.broadcast_to(_plain(x), shape)))


def take_along_axis(a, i, axis):
    return _wrap(_np.take_along_axis(_plain(a), _np.asarray(_plain(i)), axis))


def take(a, i, axis=None):
    return _wrap(_np.take(_plain(a), _plain(i), axis=axis))


def argsort(x, axis=-1, stable=True):
    return _wrap(_np.argsort(_plain(x), axis=axis, kind="stable").astype(_np.int32))


def _int_acc(x, dtype):
    if dtype is not None:
        return _canon_dtype(dtype)
    dt = _np.asarray(x).dtype
    if dt == _np.bool_ or _np.issubdtype(dt, _np.integer):
        return _np.int32
    return None


def sum(x, axis=None, dtype=None):  # noqa: A001
    x = _plain(x)
    return _wrap(_np.sum(x, axis=axis, dtype=_int_acc(x, dtype)))


def cumsum(x, axis=None, dtype=None):
    x = _plain(x)
    return _wrap(_np.cumsum(x, axis=axis, dtype=_int_acc(x, dtype)))


def _red(fn):
    return lambda x, axis=None, **k: _wrap(fn(_plain(x), axis=axis, **k))


min, max, any, all = _red(_np.min), _red(_np.max), _red(_np.any), _red(_np.all)  # noqa: A001


def argmax(x, axis=None):
    return _wrap(_np.argmax(_plain(x), axis=axis).astype(_np.int32) if axis is not None
                 else _np.int32(_np.argmax(_plain(x))))


def argmin(x, axis=None):
    return _wrap(_np.argmin(_plain(x), axis=axis).astype(_np.int32) if axis is not None
                 else _np.int32(_np.argmin(_plain(x))))


def shape(x):
    return _np.shape(x)


# ---- pytrees (NamedTuple, tuple, list, dict; None is an empty node)


def _is_node(x):
    return x is None or isinstance(x, (tuple, list, dict))


def _tree_map(f, tree, *rest):
    if tree is None:
        return None
    if isinstance(tree, dict):
        return {k: _tree_map(f, tree[k], *(r[k] for r in rest)) for k in tree}
    if isinstance(tree, tuple) and hasattr(tree, "_fields"):
        return type(tree)(*(_tree_map(f, t, *(r[i] for r in rest)) for i, t in enumerate(tree)))
    if isinstance(tree, (tuple, list)):
        return type(tree)(_tree_map(f, t, *(r[i] for r in rest)) for i, t in enumerate(tree))
    return f(tree, *rest)


def _tree_leaves(tree):
    out = []

    def visit(x):
        out.append(x)
        return x
    _tree_map(visit, tree)
    return out
