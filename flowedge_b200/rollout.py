"""Deployment loop for Diffusion Policy checkpoints on this library.

This is the host-side contract of the reference's LeRobot integration
(integrations/lerobot/src/flowedge_lerobot/diffusion.py:30-243 and
rollout.py:50-145), restated over ``flowedge_b200.Engine``:

* ``DiffusionPolicy`` reads the checkpoint's action contract from the engine
  (condition / action dims, horizon, action steps, observation steps) and
  serves the LeRobot slice of the sampled horizon: element
  ``observation_steps - 1`` for a single action, ``action_steps`` elements from
  there for a chunk.
* ``run_rollout`` runs a bounded observe -> sample -> send loop with a control
  period.  A step that takes longer than the period counts as a miss, and
  ``on_miss`` decides what the robot gets: ``hold`` re-sends the last action
  that was sent, ``drop`` sends nothing, ``raise`` raises ``DeadlineMissed``.
  ``robot.stop()`` runs on every exit path.

The engine's sample calls are synchronous (they return after the device ->
host copy), so the host clock around a step covers the device work; ``sync``
is still accepted for engines that are not.
"""

from __future__ import annotations

from dataclasses import dataclass
from math import isfinite
from time import perf_counter_ns
from typing import Any, Callable, Protocol

import numpy as np

__all__ = ["ActionContract", "DiffusionPolicy", "DeadlineMissed", "RolloutResult", "run_rollout", "ON_MISS",
           "MAX_ROLLOUT_STEPS"]

ON_MISS = ("hold", "drop", "raise")
MAX_ROLLOUT_STEPS = 100_000


class DeadlineMissed(RuntimeError):
    """A control period was exceeded with ``on_miss="raise"``."""


@dataclass(frozen=True)
class ActionContract:
    condition_dim: int
    action_dim: int
    horizon: int
    action_steps: int
    observation_steps: int

    @property
    def action_start(self) -> int:
        """First horizon element LeRobot executes (the last observed step)."""
        return self.observation_steps - 1

    @classmethod
    def from_metadata(cls, meta: dict[str, Any]) -> "ActionContract":
        keys = ("condition_dim", "action_dim", "horizon", "action_steps", "observation_steps")
        missing = [k for k in keys if k not in meta]
        if missing:
            raise ValueError(f"missing diffusion metadata: {', '.join(missing)}")
        c = cls(*(int(meta[k]) for k in keys))
        if min(c.condition_dim, c.action_dim, c.horizon, c.action_steps, c.observation_steps) <= 0:
            raise ValueError("diffusion dimensions must be positive")
        if c.action_start + c.action_steps > c.horizon:
            raise ValueError("LeRobot action slice is outside the diffusion horizon")
        return c


class _Engine(Protocol):
    @property
    def diffusion_metadata(self) -> dict[str, Any]: ...

    def sample_diffusion_into(self, condition, noise, output, steps: int = 10, scheduler: str = "ddim",
                              seed: int = 0): ...


class DiffusionPolicy:
    """LeRobot-facing adapter over a Diffusion Policy engine (no allocation per call)."""

    def __init__(self, engine: _Engine):
        self.engine = engine
        self.contract = ActionContract.from_metadata(engine.diffusion_metadata)
        self._horizon = np.empty((self.contract.horizon, self.contract.action_dim), np.float32)

    @property
    def action_dim(self) -> int:
        return self.contract.action_dim

    @property
    def noise_shape(self) -> tuple[int, int]:
        return self._horizon.shape

    def reset(self) -> None:
        """Nothing to clear: every sample call is independent."""

    def _sample(self, condition, noise, steps: int, scheduler: str, seed: int) -> None:
        condition = np.ascontiguousarray(condition, np.float32).reshape(-1)
        if condition.size != self.contract.condition_dim:
            raise ValueError(f"condition must hold {self.contract.condition_dim} float32 values")
        if np.shape(noise) != self._horizon.shape:
            raise ValueError(f"noise must have shape {self._horizon.shape}")
        if steps <= 0:
            raise ValueError("steps must be positive")
        if scheduler not in ("ddim", "ddpm"):
            raise ValueError("scheduler must be ddim or ddpm")
        self.engine.sample_diffusion_into(condition, np.ascontiguousarray(noise, np.float32), self._horizon, steps,
                                          scheduler, int(seed))

    def select_action_into(self, condition, noise, output: np.ndarray, *, steps: int = 10, scheduler: str = "ddim",
                           seed: int = 0) -> np.ndarray:
        _check_out(output, (self.contract.action_dim,))
        self._sample(condition, noise, steps, scheduler, seed)
        np.copyto(output, self._horizon[self.contract.action_start])
        return output

    def predict_action_chunk_into(self, condition, noise, output: np.ndarray, *, steps: int = 10,
                                  scheduler: str = "ddim", seed: int = 0) -> np.ndarray:
        _check_out(output, (self.contract.action_steps, self.contract.action_dim))
        self._sample(condition, noise, steps, scheduler, seed)
        s = self.contract.action_start
        np.copyto(output, self._horizon[s:s + self.contract.action_steps])
        return output


def _check_out(output, shape) -> None:
    if not (isinstance(output, np.ndarray) and output.shape == shape and output.dtype == np.float32
            and output.flags.c_contiguous):
        raise ValueError(f"output must be a C-contiguous float32 array of shape {shape}")


class Robot(Protocol):
    def reset(self) -> None: ...

    def observe(self) -> np.ndarray: ...

    def send_action(self, action: np.ndarray) -> None: ...

    def stop(self) -> None: ...


@dataclass(frozen=True)
class RolloutResult:
    steps: int
    stopped: bool
    elapsed_ms: float = 0.0
    p50_ms: float = 0.0
    p99_ms: float = 0.0
    max_ms: float = 0.0
    missed_deadlines: int = 0
    on_miss: str = "hold"


def run_rollout(policy: DiffusionPolicy, robot: Robot, encode_condition: Callable[[np.ndarray], np.ndarray], *,
                steps: int, seed: int = 0, diffusion_steps: int = 10, scheduler: str = "ddim",
                period_ms: float | None = None, on_miss: str = "hold", sync: Callable[[], None] | None = None,
                clock_ns: Callable[[], int] = perf_counter_ns) -> RolloutResult:
    """Bounded single-action control loop; see the module docstring for the miss policy.

    Step ``i`` samples with noise from ``numpy.random.default_rng(seed)`` and
    DDPM seed ``seed + i``.  ``clock_ns`` is the step clock (tests inject one).
    """
    if not 0 < steps <= MAX_ROLLOUT_STEPS:
        raise ValueError(f"steps must be from 1 through {MAX_ROLLOUT_STEPS}")
    if diffusion_steps <= 0:
        raise ValueError("diffusion_steps must be positive")
    if period_ms is not None and not (isfinite(period_ms) and period_ms > 0):
        raise ValueError("period_ms must be positive")
    if on_miss not in ON_MISS:
        raise ValueError("on_miss must be hold, drop, or raise")
    policy.reset()
    rng = np.random.default_rng(seed)
    noise = np.empty(policy.noise_shape, np.float32)
    action = np.empty(policy.action_dim, np.float32)
    last_sent = np.zeros(policy.action_dim, np.float32)
    durations = np.zeros(steps, np.int64)
    budget_ns = None if period_ms is None else period_ms * 1e6
    done = missed = 0
    t_start = clock_ns()
    try:
        robot.reset()
        for _ in range(steps):
            t0 = clock_ns()
            condition = encode_condition(robot.observe())
            rng.standard_normal(noise.shape, dtype=np.float32, out=noise)
            policy.select_action_into(condition, noise, action, steps=diffusion_steps, scheduler=scheduler,
                                      seed=seed + done)
            if sync is not None:
                sync()
            took = clock_ns() - t0
            if budget_ns is not None and took > budget_ns:
                missed += 1
                if on_miss == "raise":
                    raise DeadlineMissed(f"control period {period_ms} ms exceeded ({took / 1e6:.3f} ms)")
                if on_miss == "hold":
                    robot.send_action(last_sent)
            else:
                robot.send_action(action)
                last_sent[:] = action
            durations[done] = took
            done += 1
    finally:
        robot.stop()
    total_ms = (clock_ns() - t_start) / 1e6
    if done == 0:
        return RolloutResult(steps=0, stopped=True, elapsed_ms=total_ms, on_miss=on_miss)
    d = durations[:done] / 1e6
    p50, p99 = np.percentile(d, (50, 99))
    return RolloutResult(steps=done, stopped=True, elapsed_ms=total_ms, p50_ms=float(p50), p99_ms=float(p99),
                         max_ms=float(d.max()), missed_deadlines=missed, on_miss=on_miss)
