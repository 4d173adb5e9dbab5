"""goib2d_step_noalloc: the step for callers that cannot allocate device memory while they step (inside a CUDA
graph capture, under a host pool allocator that owns the GPU, in a loop that forbids allocation after start-up).

It must give the same states as goib2d_step, bit for bit (the tolerance of every parity test here), on consecutive
calls, and refuse batches larger than its static arena with a clear error instead of launching. This file is named
to be collected last, so a run that stops at the first failure has run every other test before it."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _leaf_ptrs(state):
    from goib2d.world import state_leaves
    leaves = state_leaves(state)
    return leaves, (C.c_void_p * len(leaves))(*[t.data_ptr() for t in leaves])


def test_noalloc_step_equals_step_on_two_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api, configs, native
    from goib2d.settings import settings_struct
    from goib2d.world import state_leaves

    sc, model, host = configs.batch("c1", 256)
    eng = api.Engine(model, host.bodies.type.shape[1], sc.action_joints, sc.action_scale)
    lib = native.load()
    ref = api.to_device(host)
    mine = api.to_device(host)
    acts = torch.from_numpy(np.random.default_rng(9).uniform(-2, 2, (256, 2)).astype(np.float32)).cuda()
    ss = settings_struct(sc.settings)
    C_, rows, n = host.contacts.pair.shape[1], host.fixtures.friction.shape[1], 256
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row: the shared arena's leftovers must not matter
        eng.step_(ref, sc.settings, configs.DT, 3, acts)
        leaves, ptrs = _leaf_ptrs(mine)
        rc = lib.goib2d_step_noalloc(eng.handle, C.addressof(ss), C.c_float(float(configs.DT)), C_, rows, n, 3, ptrs,
                                     C.c_void_p(acts.data_ptr()), C.c_void_p(stream))
        assert rc == 0, lib.goib2d_last_error()
        torch.cuda.synchronize()
        for a, b in zip(state_leaves(api.to_host(ref)), state_leaves(api.to_host(mine))):
            assert np.array_equal(a, b), f"call {call}"


def test_noalloc_after_another_models_layout():
    """The arena is shared by every model: a call on a model with a different per-world layout (c4: 23 bodies, 22
    joints, 64 contact slots) leaves other bytes at other offsets, and a following c1 call must still equal
    goib2d_step bit for bit. The no-alloc call reports no status words and no events (the log stays off)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api, configs, native
    from goib2d.settings import settings_struct
    from goib2d.world import state_leaves

    lib = native.load()
    stream = torch.cuda.current_stream().cuda_stream
    sc4, model4, host4 = configs.batch("c4", 96)
    eng4 = api.Engine(model4, host4.bodies.type.shape[1])
    dev4 = api.to_device(host4)
    _, ptrs4 = _leaf_ptrs(dev4)
    ss4 = settings_struct(sc4.settings)
    rc = lib.goib2d_step_noalloc(eng4.handle, C.addressof(ss4), C.c_float(float(configs.DT)),
                                 host4.contacts.pair.shape[1], host4.fixtures.friction.shape[1], 96, 4, ptrs4, None,
                                 C.c_void_p(stream))
    assert rc == 0, lib.goib2d_last_error()

    sc, model, host = configs.batch("c1", 200)
    eng = api.Engine(model, host.bodies.type.shape[1])
    eng.set_event_log(16)
    ref, mine = api.to_device(host), api.to_device(host)
    ss = settings_struct(sc.settings)
    eng.step_(ref, sc.settings, configs.DT, 5)
    _, ptrs = _leaf_ptrs(mine)
    rc = lib.goib2d_step_noalloc(eng.handle, C.addressof(ss), C.c_float(float(configs.DT)), host.contacts.pair.shape[1],
                                 host.fixtures.friction.shape[1], 200, 5, ptrs, None, C.c_void_p(stream))
    assert rc == 0, lib.goib2d_last_error()
    torch.cuda.synchronize()
    for a, b in zip(state_leaves(api.to_host(ref)), state_leaves(api.to_host(mine))):
        assert np.array_equal(a, b)
    events, counts = eng.events()
    assert events.shape[0] == 0 and counts.shape[0] == 0 and eng.status().shape[0] == 0
    eng.close(), eng4.close()


def test_noalloc_rejects_batches_beyond_its_arena():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api, configs, native
    from goib2d.settings import settings_struct

    sc, model, host = configs.batch("c1", 2)
    eng = api.Engine(model, host.bodies.type.shape[1])
    lib = native.load()
    dev = api.to_device(host)
    _, ptrs = _leaf_ptrs(dev)
    ss = settings_struct(sc.settings)
    too_many = 10 ** 7  # far beyond 32 MiB of arena; checked before any launch, so the small leaves are never read
    rc = lib.goib2d_step_noalloc(eng.handle, C.addressof(ss), C.c_float(0.02), host.contacts.pair.shape[1],
                                 host.fixtures.friction.shape[1], too_many, 1, ptrs, None, None)
    assert rc == -4
    assert b"static arena" in lib.goib2d_last_error()
