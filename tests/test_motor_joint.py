"""b2MotorJoint (Box2D 2.3.1's motor joint: this engine's addition, the reference engine has none, so parity with it
is unpinned). On the CPU the oracle's restatement behaves as the method promises: it drives body B to the linear and
angular offsets, and its impulses never exceed h * max force and h * max torque. On the GPU the CUDA engine equals
the oracle bit for bit."""
import numpy as np
import pytest

import oracle_lib
from goib2d import DYNAMIC, MOTOR, STATIC, Settings, WorldDef
from goib2d.world import map_state

DT = np.float32(1.0 / 60.0)


def scene(offset=(1.5, -0.5), angle=0.7, max_force=200.0, max_torque=50.0, gravity=(0.0, 0.0), mass=2.0,
          ground_angle=0.0, boxes=1):
    d = WorldDef(Settings.stock(gravity=gravity))
    g = d.add_body(STATIC, (0.3, -0.2), ground_angle)
    d.add_box(g, (4.0, 0.2), center=(0, -3))
    js = []
    for i in range(boxes):
        b = d.add_body(DYNAMIC, (0.2 * i, 0.5), 0.1 * i, mass=mass, inertia=mass / 6, allow_sleep=False)
        d.add_box(b, (0.25, 0.25))
        js.append(d.add_motor(g, b, offset, angle, max_force=max_force, max_torque=max_torque))
    return d, js


def run(d, steps, capacity=16):
    model, st = d.build(capacity)
    traj = []
    for _ in range(steps):
        st = oracle_lib.step(model, st, d.settings, DT, 1)
        traj.append(st)
    return model, traj


def test_motor_joint_reaches_its_offsets():
    """Body B's origin goes to A's origin + rot(A's angle, linear offset) and its angle to A's angle + the angular
    offset (no gravity, limits far above what the correction needs)."""
    d, _ = scene(ground_angle=0.4)
    _, traj = run(d, 240)
    st = traj[-1]
    qa = np.float64(0.4)
    want = np.array([0.3, -0.2]) + np.array([[np.cos(qa), -np.sin(qa)], [np.sin(qa), np.cos(qa)]]) @ [1.5, -0.5]
    assert np.allclose(st.bodies.xf_p[1], want, atol=1e-3), (st.bodies.xf_p[1], want)
    assert abs(float(st.bodies.a[1]) - (0.4 + 0.7)) < 1e-3
    assert np.abs(st.bodies.v[1]).max() < 1e-3 and abs(float(st.bodies.w[1])) < 1e-3


@pytest.mark.parametrize("max_force,max_torque", [(0.5, 0.05), (3.0, 0.2)])
def test_motor_joint_impulses_stay_within_their_limits(max_force, max_torque):
    d, _ = scene(max_force=max_force, max_torque=max_torque, mass=10.0)
    _, traj = run(d, 120)
    lin = np.array([np.hypot(*s.joints.impulse[0, :2]) for s in traj])
    ang = np.array([abs(float(s.joints.impulse[0, 2])) for s in traj])
    h = float(DT)
    assert lin.max() <= h * max_force * (1 + 1e-5) and ang.max() <= h * max_torque * (1 + 1e-5)
    assert lin.max() > 0.99 * h * max_force  # far from the target: the limit is reached
    # the body's speed grows by at most h * max force / mass per step
    speed = np.array([np.hypot(*s.bodies.v[1]) for s in traj])
    assert np.diff(speed).max() <= h * max_force / 10.0 * (1 + 1e-4)


def test_motor_joint_holds_a_body_against_gravity():
    d, _ = scene(gravity=(0.0, -10.0), offset=(0.0, 1.0), angle=0.0, max_force=100.0)
    _, traj = run(d, 300)
    st = traj[-1]
    assert np.allclose(st.bodies.xf_p[1], [0.3, 0.8], atol=0.02), st.bodies.xf_p[1]
    # the joint carries the weight: linear impulse per step = m g h upwards
    assert abs(float(st.joints.impulse[0, 1]) - 2.0 * 10.0 * float(DT)) < 1e-3


def test_motor_joint_row_layout():
    """The joint row holds the motor joint's parameters (see WorldDef.add_motor)."""
    d, _ = scene(offset=(0.25, 0.75), angle=-0.3, max_force=7.0, max_torque=3.0)
    model, st = d.build(8)
    assert int(model.joint_type[0]) == MOTOR
    j = st.joints
    assert (float(j.lower[0]), float(j.upper[0]), float(j.motor_speed[0])) == (0.25, 0.75, np.float32(-0.3))
    assert (float(j.max_motor[0]), float(j.frequency[0]), float(j.damping[0])) == (3.0, 7.0, np.float32(0.3))


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [1, 2])
def test_gpu_motor_joints_match_oracle(mode):
    """Batches of motor-jointed boxes that fall, collide and are driven to per-world offsets (the joint row of each
    world set differently) equal the oracle bit for bit."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api
    from test_oracle import assert_states_equal
    d, _ = scene(gravity=(0.0, -10.0), boxes=4, max_force=30.0, max_torque=5.0)
    model, st = d.build(24)
    n = 48
    host = map_state(lambda x: np.ascontiguousarray(np.repeat(np.asarray(x)[None], n, 0)), st)
    rng = np.random.default_rng(17)
    host.joints.lower[...] = rng.uniform(-2, 2, host.joints.lower.shape).astype(np.float32)
    host.joints.upper[...] = rng.uniform(-3, 1, host.joints.upper.shape).astype(np.float32)
    host.joints.motor_speed[...] = rng.uniform(-3, 3, host.joints.motor_speed.shape).astype(np.float32)
    dyn = (host.bodies.type == 2)[..., None]
    host.bodies.v[...] = np.where(dyn, rng.normal(0, 1.0, host.bodies.v.shape), host.bodies.v).astype(np.float32)
    eng = api.Engine(model, host.bodies.type.shape[1])
    try:
        eng.set_step_mode(mode)
        dev = api.to_device(host)
        eng.step_(dev, d.settings, DT, n_steps=90)
        got = api.to_host(dev)
    finally:
        eng.close()
    want = oracle_lib.step(model, host, d.settings, DT, 90, threads=8)
    assert_states_equal(got, want, f"motor mode {mode}")
