"""rot_of's fast path (double-precision sin / cos with a rounding test) against the float-float evaluation the
reference defines (goi_jax/box2d/math2d.py:218-316, restated as rot_of_ff): equal bit for bit on EVERY float32
argument. The sweep covers all 2^32 bit patterns (non-finite ones excepted) and takes seconds on a B200."""
import ctypes as C
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
LIB = Path(__file__).resolve().parents[1] / "getting-over-it-rl_b200" / "goib2d" / "libgoib2d_rotcheck.so"


def _sweep(lo, hi, stride=1):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    assert LIB.exists(), f"{LIB} not built (run csrc/build.sh)"
    lib = C.CDLL(str(LIB))
    out = (C.c_ulonglong * 260)()
    rc = lib.goib2d_rot_check(C.c_uint64(lo), C.c_uint64(hi), C.c_uint64(stride), out)
    assert rc == 0, f"CUDA error {rc}"
    return out


def test_rot_fast_equals_float_float_on_every_float():
    out = _sweep(0, 1 << 32)
    non_finite = 2 * (1 << 23)  # exponent field all ones, both signs
    assert out[0] == (1 << 32) - non_finite
    assert out[1] == 0, f"{out[1]} arguments differ, the lowest bit pattern {out[3]:#010x}"


def test_rot_fast_takes_the_fast_path_for_ordinary_angles():
    lo, hi = 0x3c000000, 0x41200000  # [2^-7, 10) rad: the angles bodies have
    out = _sweep(lo, hi)
    assert out[1] == 0
    assert out[2] < 0.01 * out[0], f"{out[2]} of {out[0]} arguments fell back to the float-float path"
