"""The C-ABI library loads on a CPU-only host and exports every function include/goib2d.h declares (no compute)."""
import ctypes
import re
from pathlib import Path

import pytest

from goib2d import native

ROOT = Path(__file__).resolve().parents[1]


def declared():
    text = (ROOT / "include" / "goib2d.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char \*)\s*\*?(goib2d_\w+)\(", text, re.M)))


def test_header_declares_the_entry_points():
    names = declared()
    for n in ("goib2d_version", "goib2d_last_error", "goib2d_model_create", "goib2d_model_destroy", "goib2d_step",
              "goib2d_status", "goib2d_leaf_elems", "goib2d_leaf_dtype", "goib2d_model_set_action_map"):
        assert n in names


def test_library_exports_every_declared_symbol():
    if not native.lib_path().exists():
        pytest.skip("libgoib2d.so not built (run __graft_entry__.build())")
    lib = ctypes.CDLL(str(native.lib_path()))
    for n in declared():
        assert hasattr(lib, n), n
    lib = native.load()
    assert lib.goib2d_version() == 2
    assert lib.goib2d_kernels_per_step(None, 4096) < 0  # a null model is an error, not a count
    assert lib.goib2d_launches(None, 4096, 10) < 0
    assert lib.goib2d_step_seq(None, None, 0.02, 8, 1, 1, 1, None, None, 0, None) == -1
    assert lib.goib2d_set_step_mode(None, 1) < 0 and b"null" in lib.goib2d_last_error()
    assert lib.goib2d_set_state_staging(None, 4096) < 0 and b"null" in lib.goib2d_last_error()
    for leaf in range(71):  # the leaf table agrees with the Python one (no device needed)
        B, rows, J, C = 5, 7, 3, 11
        spec = native.leaf_spec(B, rows, J, C)[leaf]
        import numpy as np
        assert lib.goib2d_leaf_elems(leaf, B, rows, J, C) == int(np.prod(spec[1]))
        assert lib.goib2d_leaf_dtype(leaf) == {np.dtype(np.float32): 0, np.dtype(np.int32): 1,
                                              np.dtype(np.bool_): 2}[spec[2]]


def test_model_create_rejects_bad_descriptors_without_a_gpu():
    """Argument checks run before any device call."""
    if not native.lib_path().exists():
        pytest.skip("libgoib2d.so not built")
    lib = native.load()
    d = native.ModelDesc()
    d.n_bodies, d.n_fixtures = -1, 0
    h = ctypes.c_void_p()
    assert lib.goib2d_model_create(ctypes.byref(d), ctypes.byref(h)) == -1
    assert b"negative" in lib.goib2d_last_error()


def test_settings_struct_is_25_words():
    """The FFI binding passes goib2d_settings as its 25 32-bit words; the struct must stay that."""
    import numpy as np
    from goib2d.settings import Settings, SettingsC, settings_struct
    assert ctypes.sizeof(SettingsC) == 25 * 4
    words = np.frombuffer(bytes(settings_struct(Settings.game())), np.int32)
    back = SettingsC.from_buffer_copy(words.tobytes())
    assert back.velocity_iterations == 300 and back.position_iterations == 30 and back.continuous_physics == 1
