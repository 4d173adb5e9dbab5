"""The scene build on the device: goib2d_candidate_pairs gives the host builder's candidate list (same pairs, same
order, same orientation) on the benchmark levels, the edge scenes and a scene exercising every exclusion rule."""
import numpy as np
import pytest

import edge_scenes
from goib2d.settings import Settings
from goib2d.world import DYNAMIC, STATIC, WorldDef

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _rules_scene(layers=False):
    d = WorldDef(Settings.stock(), layer_masks=[(0xFFFFFFFF ^ (1 << 3)) if k == 2 else 0xFFFFFFFF for k in range(32)]
                 if layers else None)
    g = d.add_body(STATIC)
    d.add_box(g, (5.0, 0.5))
    d.add_edge(g, (-5.0, 1.0), (5.0, 1.0))
    d.add_circle(g, 0.5, (3.0, 3.0), sensor=True)
    bodies = [d.add_body(DYNAMIC, (float(i), 2.0), mass=1.0, inertia=0.1) for i in range(6)]
    d.add_circle(bodies[0], 0.3, group=-2)
    d.add_circle(bodies[1], 0.3, group=-2)           # same negative group: never
    d.add_box(bodies[2], (0.2, 0.2), group=3, layer=2)
    d.add_box(bodies[3], (0.2, 0.2), group=3, layer=3)  # same positive group: always (layers: 2 vs 3 filtered)
    d.add_polygon(bodies[4], [(-0.2, -0.2), (0.3, -0.1), (0.0, 0.3)], category=2, mask=0xFFFD)  # not with category 2
    d.add_box(bodies[4], (0.1, 0.1), center=(0.3, 0.0), category=2, mask=0xFFFF)
    d.add_circle(bodies[5], 0.2, sensor=True)
    d.add_revolute(bodies[0], bodies[2])                # joined, no collideConnected
    d.add_revolute(bodies[1], bodies[3], collide=True)  # joined, collideConnected
    return d


def _defs():
    from goib2d import configs
    out = [("rules", _rules_scene()), ("rules_layers", _rules_scene(True))]
    for cfg in ("c0", "c1", "c1e", "c3e", "c4"):
        sc = configs.scene(cfg, n=2)
        out.append((cfg, sc.world_def(0)))
    for name, fn in edge_scenes.SCENES.items():
        out.append((name, fn()))
    return out


def test_device_candidate_pairs_equal_the_host_list():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    for name, d in _defs():
        host = d.candidate_pairs()
        dev = d.candidate_pairs(device=True)
        assert dev == host, name
    assert len(_rules_scene().candidate_pairs()) > 0
