"""World constants: Box2D 2.3.1's b2Settings plus Getting Over It's Physics2D values.

Mirrors goi_jax/box2d/settings.py (reference): the same field names, defaults and class methods, so code written
against `goi_jax.box2d.Settings` runs unchanged. Every float is the float32 value Box2D holds, computed the way
b2Settings.h computes it (e.g. `2.0f / 180.0f * b2_pi`, left to right in float32; reference settings.py:99-106).

`Settings` is frozen and hashable. `settings_struct()` packs it into the C struct `goib2d_settings`
(include/goib2d.h) that the CUDA library reads.
"""
import ctypes
from dataclasses import dataclass, fields, replace

import numpy as np

F32 = np.float32

# b2Settings.h compile-time constants (reference settings.py:84-96)
PI = F32(3.14159265359)
EPSILON = F32(np.finfo(np.float32).eps)
MAX_FLOAT = F32(np.finfo(np.float32).max)
MAX_MANIFOLD_POINTS = 2
MAX_POLYGON_VERTICES = 8
AABB_EXTENSION = F32(0.1)
AABB_MULTIPLIER = F32(2.0)
MAX_SUB_STEPS = 8
MAX_TOI_CONTACTS = 32
MAX_CONDITION_NUMBER = F32(1000.0)
K_TOL = F32(0.1)


def deg2rad(deg):
    """Unity's Mathf.Deg2Rad product in float32 (reference settings.py:99-101)."""
    return F32(F32(deg) * F32(0.0174532924))


def _b2_angle(deg):
    """`deg / 180.0f * b2_pi` evaluated left to right in float32 (the b2Settings.h macro form)."""
    q = F32(F32(deg) / F32(180.0))
    return F32(q * PI)


@dataclass(frozen=True)
class Settings:
    """Defaults are stock Box2D 2.3.1; `Settings.game()` is Getting Over It (reference settings.py:109-163)."""
    gravity: tuple = (F32(0.0), F32(-10.0))
    velocity_iterations: int = 8
    position_iterations: int = 3
    linear_slop: F32 = F32(0.005)
    angular_slop: F32 = _b2_angle(2.0)
    polygon_radius: F32 = F32(F32(2.0) * F32(0.005))
    velocity_threshold: F32 = F32(1.0)
    max_linear_correction: F32 = F32(0.2)
    max_angular_correction: F32 = _b2_angle(8.0)
    max_translation: F32 = F32(2.0)
    max_rotation: F32 = F32(F32(0.5) * PI)
    baumgarte: F32 = F32(0.2)
    toi_baumgarte: F32 = F32(0.75)
    time_to_sleep: F32 = F32(0.5)
    linear_sleep_tolerance: F32 = F32(0.01)
    angular_sleep_tolerance: F32 = _b2_angle(2.0)
    clamps_per_second: bool = False
    allow_sleep: bool = True
    warm_starting: bool = True
    continuous_physics: bool = False
    unity_toi: bool = False
    toi_tie_oldest: bool = False
    auto_clear_forces: bool = True
    revolute_v24: bool = True
    # Kept for signature compatibility with the reference (its "xla" / "pallas" switch). This engine has one path,
    # the CUDA kernels of libgoib2d; any value runs it.
    solver: str = "cuda"

    @classmethod
    def stock(cls, **kw):
        return replace(cls(), **{k: _cast(v) for k, v in kw.items()})

    @classmethod
    def game(cls, **kw):
        """Getting Over It's Physics2D settings (reference settings.py:154-163)."""
        s = cls(gravity=(F32(0.0), F32(-30.0)), velocity_iterations=300, position_iterations=30,
                velocity_threshold=F32(1.0), max_linear_correction=F32(0.2), max_angular_correction=deg2rad(8),
                max_translation=F32(100.0), max_rotation=deg2rad(360), baumgarte=F32(0.4), toi_baumgarte=F32(0.75),
                time_to_sleep=F32(0.5), linear_sleep_tolerance=F32(0.01), angular_sleep_tolerance=deg2rad(2),
                linear_slop=F32(0.005), polygon_radius=F32(0.01), continuous_physics=True, unity_toi=True,
                toi_tie_oldest=True)
        return replace(s, **{k: _cast(v) for k, v in kw.items()})

    def to_dict(self):
        out = {}
        for f in fields(self):
            v = getattr(self, f.name)
            out[f.name] = [float(x) for x in v] if isinstance(v, tuple) else (
                float(v) if isinstance(v, (float, np.floating)) else v)
        return out

    @classmethod
    def from_dict(cls, d):
        kw = {}
        for f in fields(cls):
            if f.name in d:
                v = d[f.name]
                kw[f.name] = tuple(F32(x) for x in v) if isinstance(v, (list, tuple)) else _cast(v)
        return cls(**kw)


def _cast(v):
    if isinstance(v, str):
        return v
    if isinstance(v, (bool, np.bool_)):
        return bool(v)
    if isinstance(v, (int, np.integer)):
        return int(v)
    if isinstance(v, (tuple, list)):
        return tuple(F32(x) for x in v)
    return F32(v)


class SettingsC(ctypes.Structure):
    """`goib2d_settings` of include/goib2d.h, field for field."""
    _fields_ = [(n, ctypes.c_float) for n in (
        "gravity_x", "gravity_y", "linear_slop", "angular_slop", "polygon_radius", "velocity_threshold",
        "max_linear_correction", "max_angular_correction", "max_translation", "max_rotation", "baumgarte",
        "toi_baumgarte", "time_to_sleep", "linear_sleep_tolerance", "angular_sleep_tolerance")] + \
        [(n, ctypes.c_int32) for n in (
            "velocity_iterations", "position_iterations", "clamps_per_second", "allow_sleep", "warm_starting",
            "continuous_physics", "unity_toi", "toi_tie_oldest", "auto_clear_forces", "revolute_v24")]


def settings_struct(s: Settings) -> SettingsC:
    c = SettingsC()
    c.gravity_x, c.gravity_y = float(s.gravity[0]), float(s.gravity[1])
    for n in ("linear_slop", "angular_slop", "polygon_radius", "velocity_threshold", "max_linear_correction",
              "max_angular_correction", "max_translation", "max_rotation", "baumgarte", "toi_baumgarte",
              "time_to_sleep", "linear_sleep_tolerance", "angular_sleep_tolerance"):
        setattr(c, n, float(getattr(s, n)))
    for n in ("velocity_iterations", "position_iterations", "clamps_per_second", "allow_sleep", "warm_starting",
              "continuous_physics", "unity_toi", "toi_tie_oldest", "auto_clear_forces", "revolute_v24"):
        setattr(c, n, int(getattr(s, n)))
    return c
