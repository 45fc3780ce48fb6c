"""Host-side deployment contract (flowedge_b200/rollout.py): the LeRobot action
slice and the control-period miss policy (`--on-miss hold|drop|raise`) of the
reference's rollout loop (integrations/lerobot/src/flowedge_lerobot/rollout.py:95-124),
driven with a fake engine that spends time on a fake clock, and a fake robot
(no GPU)."""

import numpy as np
import pytest

from flowedge_b200.rollout import ControlLoop, DeadlineMissed, DiffusionPolicy, MissPolicy, run_rollout

META = {"condition_dim": 4, "action_dim": 2, "horizon": 6, "action_steps": 3, "observation_steps": 2}


class FakeClock:
    """Nanosecond clock that only moves when a fake sample call spends time."""

    def __init__(self):
        self.t = 0

    def __call__(self):
        return self.t


class FakeEngine:
    """Horizon row t is filled with (seed * 10 + t, condition[0]); call i takes
    durations_ms[i] on the fake clock."""

    diffusion_metadata = META

    def __init__(self, clock=None, durations_ms=()):
        self.calls = []
        self.clock, self.durations = clock, list(durations_ms)

    def sample_diffusion_into(self, condition, noise, output, steps=10, scheduler="ddim", seed=0):
        if self.clock is not None and len(self.calls) < len(self.durations):
            self.clock.t += int(self.durations[len(self.calls)] * 1e6)
        self.calls.append((steps, scheduler, seed))
        output[:, 0] = seed * 10 + np.arange(output.shape[0])
        output[:, 1] = condition[0]


class FakeRobot:
    def __init__(self):
        self.sent, self.events = [], []

    def reset(self):
        self.events.append("reset")

    def observe(self):
        return np.full(4, len(self.sent), np.float32)

    def send_action(self, action):
        self.sent.append(np.array(action))

    def stop(self):
        self.events.append("stop")


def test_action_slice_is_the_lerobot_contract():
    eng = FakeEngine()
    pol = DiffusionPolicy(eng)
    assert pol.contract.action_start == 1 and pol.noise_shape == (6, 2)
    out = np.empty(2, np.float32)
    pol.select_action_into(np.arange(4, dtype=np.float32), np.zeros((6, 2), np.float32), out, seed=3)
    np.testing.assert_array_equal(out, [31, 0])  # horizon element observation_steps - 1
    chunk = np.empty((3, 2), np.float32)
    pol.predict_action_chunk_into(np.ones(4, np.float32), np.zeros((6, 2), np.float32), chunk, seed=0)
    np.testing.assert_array_equal(chunk[:, 0], [1, 2, 3])
    with pytest.raises(ValueError):
        pol.select_action_into(np.zeros(3, np.float32), np.zeros((6, 2), np.float32), out)
    with pytest.raises(ValueError):
        DiffusionPolicy(type("E", (), {"diffusion_metadata": dict(META, observation_steps=5)})())


@pytest.mark.parametrize("on_miss", ["hold", "drop"])
def test_missed_periods_hold_or_drop(on_miss):
    robot = FakeRobot()
    clock = FakeClock()
    engine = FakeEngine(clock, [1, 9, 1, 9, 9, 1])  # ms per step; period 5 ms -> steps 1, 3, 4 miss
    res = run_rollout(DiffusionPolicy(engine), robot, lambda obs: obs, steps=6, period_ms=5.0,
                      on_miss=on_miss, clock_ns=clock)
    assert res.steps == 6 and res.missed_deadlines == 3 and robot.events == ["reset", "stop"]
    if on_miss == "hold":
        assert len(robot.sent) == 6
        # a miss re-sends the last action that was sent (seed 0 and seed 2 actions)
        np.testing.assert_array_equal(robot.sent[1], robot.sent[0])
        np.testing.assert_array_equal(robot.sent[3], robot.sent[2])
        np.testing.assert_array_equal(robot.sent[4], robot.sent[2])
        assert robot.sent[5][0] == 51
    else:
        assert [a[0] for a in robot.sent] == [1, 21, 51]
    assert res.max_ms == pytest.approx(9.0) and res.p50_ms == pytest.approx(5.0)


def test_raise_stops_the_robot():
    robot = FakeRobot()
    clock = FakeClock()
    with pytest.raises(DeadlineMissed):
        run_rollout(DiffusionPolicy(FakeEngine(clock, [1, 7, 1, 1])), robot, lambda o: o, steps=4, period_ms=5.0,
                    on_miss="raise", clock_ns=clock)
    assert robot.events == ["reset", "stop"] and len(robot.sent) == 1


def test_seeds_noise_and_argument_checks():
    eng = FakeEngine()
    run_rollout(DiffusionPolicy(eng), FakeRobot(), lambda o: o, steps=3, seed=7, diffusion_steps=4,
                scheduler="ddpm")
    assert eng.calls == [(4, "ddpm", 7), (4, "ddpm", 8), (4, "ddpm", 9)]
    for kw in (dict(steps=0), dict(steps=2, period_ms=0.0), dict(steps=2, on_miss="skip"),
               dict(steps=2, diffusion_steps=0)):
        with pytest.raises(ValueError):
            run_rollout(DiffusionPolicy(eng), FakeRobot(), lambda o: o, **kw)


def test_hold_before_any_send_holds_zeros_and_report_fields():
    robot = FakeRobot()
    clock = FakeClock()
    loop = ControlLoop(DiffusionPolicy(FakeEngine(clock, [8, 1, 8])), robot, lambda o: o, period_ms=5.0,
                       clock_ns=clock)
    rep = loop.run(3, seed=2)
    np.testing.assert_array_equal(robot.sent[0], [0, 0])  # nothing was sent yet: the held action is zeros
    assert robot.sent[1][0] == 31 and robot.sent[2][0] == 31  # step 1 (seed 3) sent, then held
    assert rep.steps == 3 and rep.missed_deadlines == 2 and rep.on_miss == "hold" and rep.stopped
    assert rep.latencies_ns.tolist() == [8_000_000, 1_000_000, 8_000_000]
    assert rep.elapsed_ms == pytest.approx(17.0) and rep.max_ms == pytest.approx(8.0)
    assert MissPolicy("drop") is MissPolicy.DROP
