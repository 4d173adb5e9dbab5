"""Host logic: the builder (goib2d.WorldDef) against the reference's (golden builder-call logs and built states),
Settings against the reference's values, the workload generators, the C-ABI leaf table. CPU only."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import goldens
from goib2d import Settings, WorldDef, configs, native
from goib2d.world import (Model, compact_model, compact_state, expand_state, leaf_names, state_leaves)
from test_oracle import assert_states_equal

ROOT = Path(__file__).resolve().parents[1]
NAMES = goldens.names()


def replay(g):
    d = WorldDef(g.settings, layer_masks=g.meta.get("layer_masks"))
    for name, args, kwargs in g.meta["calls"]:
        getattr(d, name)(*[tuple(a) if isinstance(a, list) else a for a in args],
                         **{k: (tuple(v) if isinstance(v, list) and k != "vertices" else v) for k, v in kwargs.items()})
    return d


@pytest.mark.parametrize("name", NAMES)
def test_builder_matches_reference(name):
    g = goldens.Golden(name)
    d = replay(g)
    model, state = d.build(g.capacity)
    if g.meta["compact"]:
        model = compact_model(model, state)
        state = compact_state(model, state)
    for f in Model._fields:
        ref = getattr(g.model, f)
        if ref is None or f.startswith("scan_"):
            continue
        mine = np.asarray(getattr(model, f))
        assert mine.shape == ref.shape and np.array_equal(mine.astype(ref.dtype), ref), f
    assert_states_equal(state, g.state(0), name)


def test_settings_match_reference():
    """Settings.game() / Settings() are the reference's values bit for bit (as recorded in the golden metadata)."""
    for name, mine in (("game_pile", Settings.game()), ("stock_pile", Settings())):
        ref = goldens.Golden(name).meta["settings"]
        for k, v in mine.to_dict().items():
            if k == "solver":
                continue
            rv = ref[k]
            if isinstance(v, list):
                assert [np.float32(x) for x in v] == [np.float32(x) for x in rv], k
            elif isinstance(v, float):
                assert np.float32(v).tobytes() == np.float32(rv).tobytes(), k
            else:
                assert v == rv, k


@pytest.mark.parametrize("cfg,world", [("c0", 0), ("c1", 0), ("c1", 1), ("c3", 0), ("c4", 0)])
def test_batch_generator_equals_per_world_builds(cfg, world):
    """configs.batch builds each world's State like a full WorldDef build of that world (the golden's s0)."""
    g = goldens.Golden(f"{cfg}_w{world}")
    sc, model, state = configs.batch(cfg, 2)
    one = type(state)(*[type(getattr(state, f))(*[x[world] for x in getattr(state, f)])
                        if isinstance(getattr(state, f), tuple) else getattr(state, f)[world] for f in state._fields])
    assert_states_equal(one, g.state(0), cfg)
    assert np.array_equal(model.pair_a, g.model.pair_a) and np.array_equal(model.fixture_slot, g.model.fixture_slot)


def test_compact_roundtrip():
    sc, model, state = configs.batch("c1", 3)
    full = expand_state(model, state)
    assert full.fixtures.fat.shape[1] == model.fixture_body.shape[0]
    again = compact_state(model, full)
    for a, b in zip(state_leaves(again), state_leaves(state)):
        assert np.array_equal(a, b)


def test_leaf_table_matches_header():
    """goib2d/native.py's leaf order and include/goib2d.h's enum agree."""
    text = (ROOT / "include" / "goib2d.h").read_text()
    start = text.index("enum goib2d_leaf {")
    body = text[start:text.index("GOIB2D_NUM_LEAVES", start)]
    enum = re.findall(r"GOIB2D_([A-Z0-9_]+)", body)
    assert len(enum) == len(leaf_names()) == 71
    norm = lambda s: s.replace(".", "_").upper()  # noqa: E731
    prefix = {"BODIES": "B", "FIXTURES": "F", "JOINTS": "J", "CONTACTS": "C", "TOI": "T"}
    for e, n in zip(enum, leaf_names()):
        grp, _, field = n.partition(".")
        want = (prefix[grp.upper()] + "_" + norm(field)) if field else norm(grp)
        assert e == want, (e, n)


def test_state_bytes_formula():
    """Per-world leaf bytes match the element table for a c1 world (rows = Fd)."""
    sc, model, state = configs.batch("c1", 2)
    B, rows, J, C = 4, 3, 2, 48
    spec = native.leaf_spec(B, rows, J, C)
    for (name, shape, dt), leaf in zip(spec, state_leaves(state)):
        assert leaf.shape[1:] == shape and leaf.dtype == dt, name
