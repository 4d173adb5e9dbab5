"""goib2d: batched Box2D 2.3.1 world step on NVIDIA B200 - a drop-in for goi_jax.box2d's step.

    import goib2d as jb
    d = jb.WorldDef(jb.Settings.game())            # the reference's builder calls and defaults
    g = d.add_body(jb.STATIC); d.add_box(g, (10, 0.5), friction=1.0)
    b = d.add_body(jb.DYNAMIC, (0, 1.2), 0.3, mass=2, inertia=1 / 3); d.add_box(b, (0.5, 0.5))
    model, state = d.build(contact_capacity=16)
    batch = jb.to_device(jb.broadcast(state, 4096))            # (N, ...) leaves in HBM
    batch = jb.step(model, batch, d.settings, jb.GAME_DT)       # b2World::Step of every world, CUDA kernels

Same names as the reference package (goi_jax/box2d/__init__.py:62-68): WorldDef, Settings (.stock / .game), Model,
State, step(model, state, settings, dt, axis_name=None), GAME_DT, the body / joint type constants, and
world.compact_model / compact_state / expand_state. The step runs in libgoib2d.so (include/goib2d.h); there is no
CPU path behind it.
"""
import numpy as np

from .settings import Settings
from .world import (DYNAMIC, KINEMATIC, MOTOR, PRISMATIC, REVOLUTE, STATIC, WELD, Model, State, WorldDef,
                    compact_model, compact_state, expand_state)

GAME_DT = np.float32(0.008333334)  # Time.fixedDeltaTime as float32 (reference __init__.py:68)


def __getattr__(name):
    # the device API imports torch; load it only when used
    if name in ("step", "step_", "to_device", "to_host", "broadcast", "Engine", "build"):
        from . import api
        return getattr(api, name)
    raise AttributeError(name)


__all__ = ["Settings", "WorldDef", "Model", "State", "step", "step_", "GAME_DT", "STATIC", "KINEMATIC", "DYNAMIC",
           "REVOLUTE", "PRISMATIC", "WELD", "MOTOR", "compact_model", "compact_state", "expand_state", "to_device", "to_host",
           "broadcast", "Engine"]
