"""Load the golden vectors of tests/golden/*.npz (made by tests/golden/make_golden.py from the reference engine)."""
import json
from pathlib import Path

import numpy as np

from goib2d.world import Model, leaf_names, state_from_leaves

GOLDEN = Path(__file__).resolve().parent / "golden"


def names():
    return sorted(p.stem for p in GOLDEN.glob("*.npz"))


class Golden:
    def __init__(self, name):
        z = np.load(GOLDEN / f"{name}.npz")
        self.meta = json.loads(str(z["meta"]))
        self.name = name
        self.model = Model(**{f: (z[f"model.{f}"] if f"model.{f}" in z else None) for f in Model._fields})
        self.traj = {leaf: z[f"traj.{leaf}"] for leaf in leaf_names()}
        self.checkpoints = self.meta["checkpoints"]

    def state(self, k=0, batch=None):
        """The reference's State after checkpoint step k; batch: a leading world axis of that size (copies)."""
        i = self.checkpoints.index(k)
        leaves = [self.traj[n][i] for n in leaf_names()]
        if batch is not None:
            leaves = [np.ascontiguousarray(np.broadcast_to(x, (batch,) + x.shape)) for x in leaves]
        else:
            leaves = [x.copy() for x in leaves]
        return state_from_leaves(leaves)

    @property
    def settings(self):
        from goib2d.settings import Settings
        return Settings.from_dict(self.meta["settings"])

    @property
    def dt(self):
        return np.float32(self.meta["dt"])

    @property
    def capacity(self):
        return int(self.meta["capacity"])

    @property
    def n_bodies(self):
        return int(self.traj["bodies.type"].shape[1])

    @property
    def rows(self):
        return int(self.traj["fixtures.friction"].shape[1])
