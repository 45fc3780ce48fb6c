"""The deployment loop (flowedge_b200/rollout.py) on the real engine: PushT
U-Net, DDIM-10; each sent action is horizon element observation_steps - 1 of a
direct sample call with the same noise."""

import numpy as np
import pytest

from flowedge_b200 import Engine
from flowedge_b200 import checkpoint as ck
from flowedge_b200.rollout import DiffusionPolicy, run_rollout

pytestmark = pytest.mark.gpu


class Robot:
    def __init__(self):
        self.sent, self.stopped = [], False

    def reset(self):
        pass

    def observe(self):
        return np.random.default_rng(len(self.sent)).standard_normal(132).astype(np.float32)

    def send_action(self, action):
        self.sent.append(np.array(action))

    def stop(self):
        self.stopped = True


def test_rollout_on_pusht(tmp_path):
    t, m = ck.diffusion_tensors(ck.PUSHT, seed=3)
    path = tmp_path / "pusht.safetensors"
    ck.write_checkpoint(path, t, metadata=m)
    e = Engine(path, threads=0, device=0)
    policy = DiffusionPolicy(e)
    robot = Robot()
    res = run_rollout(policy, robot, lambda obs: obs, steps=5, seed=11, period_ms=1000.0)
    assert res.steps == 5 and res.missed_deadlines == 0 and robot.stopped and len(robot.sent) == 5
    print(f"PushT rollout step p50 {res.p50_ms:.2f} ms, max {res.max_ms:.2f} ms")
    rng = np.random.default_rng(11)
    start = policy.contract.action_start
    for i in range(5):
        noise = rng.standard_normal(policy.noise_shape, dtype=np.float32)
        cond = np.random.default_rng(i).standard_normal(132).astype(np.float32)
        np.testing.assert_array_equal(robot.sent[i], e.sample_diffusion(cond, noise, 10, "ddim", 11 + i)[start])
    e.close()
