"""Deployment loop for Diffusion Policy checkpoints on this library.

This is the host-side contract of the reference's LeRobot integration
(integrations/lerobot/src/flowedge_lerobot/diffusion.py:30-243 and
rollout.py:50-145), restated over ``flowedge_b200.Engine``:

* ``DiffusionPolicy`` reads the checkpoint's action contract from the engine
  (condition / action dims, horizon, action steps, observation steps) and
  serves the LeRobot slice of the sampled horizon: element
  ``observation_steps - 1`` for a single action, ``action_steps`` elements from
  there for a chunk.
* ``ControlLoop`` (and ``run_rollout`` over it) runs a bounded observe ->
  sample -> dispatch loop with a control period.  A step that takes longer
  than the period counts as a miss, and the ``on_miss`` policy (``MissPolicy``)
  decides what the robot gets: ``hold`` re-sends the last action that was
  sent, ``drop`` sends nothing, ``raise`` raises ``DeadlineMissed``.
  ``robot.stop()`` runs on every exit path.  This is the reference's
  ``--on-miss hold|drop|raise`` contract (rollout.py:95-124); the loop itself
  is this library's own.

The engine's sample calls are synchronous (they return after the device ->
host copy), so the host clock around a step covers the device work; ``sync``
is still accepted for engines that are not.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from math import isfinite
from time import perf_counter_ns
from typing import Any, Callable, Protocol

import numpy as np

__all__ = ["ActionContract", "ControlLoop", "DiffusionPolicy", "DeadlineMissed", "LoopReport", "MissPolicy",
           "run_rollout", "ON_MISS", "MAX_ROLLOUT_STEPS"]

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


class MissPolicy(str, Enum):
    """What the robot receives when a control step overruns its period."""

    HOLD = "hold"  # the action sent most recently, again (zeros before the first send)
    DROP = "drop"  # nothing this period
    RAISE = "raise"  # DeadlineMissed, after robot.stop()


@dataclass
class LoopReport:
    """Per-step latencies of a finished loop (the host clock around observe ->
    sample -> dispatch, device work included) and its miss count."""

    latencies_ns: np.ndarray
    missed_deadlines: int
    on_miss: str
    elapsed_ms: float
    stopped: bool = True

    @property
    def steps(self) -> int:
        return int(self.latencies_ns.size)

    def _quantile_ms(self, q: float) -> float:
        return float(np.percentile(self.latencies_ns, q)) / 1e6 if self.steps else 0.0

    @property
    def p50_ms(self) -> float:
        return self._quantile_ms(50)

    @property
    def p99_ms(self) -> float:
        return self._quantile_ms(99)

    @property
    def max_ms(self) -> float:
        return float(self.latencies_ns.max()) / 1e6 if self.steps else 0.0


class ControlLoop:
    """A fixed-period observe -> sample -> dispatch loop over a policy.

    All buffers (noise, the sampled action, the held action, the latency log)
    are allocated here, once; a step allocates nothing on the host.  The step
    clock is injectable (``clock_ns``) so the miss policy can be tested without
    real time.  ``sync`` is called after sampling for engines whose calls
    return before the device finishes (this library's do not).
    """

    def __init__(self, policy: DiffusionPolicy, robot: Robot, encode_condition: Callable[[np.ndarray], np.ndarray],
                 *, period_ms: float | None = None, on_miss: str = "hold", sync: Callable[[], None] | None = None,
                 clock_ns: Callable[[], int] = perf_counter_ns):
        if period_ms is not None and not (isfinite(period_ms) and period_ms > 0):
            raise ValueError("period_ms must be positive")
        try:
            self.on_miss = MissPolicy(on_miss)
        except ValueError:
            raise ValueError("on_miss must be hold, drop, or raise") from None
        self.policy, self.robot, self.encode = policy, robot, encode_condition
        self.period_ns = None if period_ms is None else int(period_ms * 1e6)
        self.sync, self.clock = sync, clock_ns
        self._noise = np.empty(policy.noise_shape, np.float32)
        self._action = np.empty(policy.action_dim, np.float32)
        self._held = np.zeros(policy.action_dim, np.float32)

    def _late(self, took_ns: int) -> bool:
        return self.period_ns is not None and took_ns > self.period_ns

    def _dispatch(self, late: bool, took_ns: int) -> None:
        if not late:
            self.robot.send_action(self._action)
            np.copyto(self._held, self._action)
        elif self.on_miss is MissPolicy.HOLD:
            self.robot.send_action(self._held)
        elif self.on_miss is MissPolicy.RAISE:
            raise DeadlineMissed(f"control period {self.period_ns / 1e6:g} ms exceeded "
                                 f"({took_ns / 1e6:.3f} ms)")

    def run(self, steps: int, *, seed: int = 0, diffusion_steps: int = 10, scheduler: str = "ddim") -> LoopReport:
        """Run `steps` control steps.  Step i draws its initial noise from
        ``numpy.random.default_rng(seed)`` (one stream for the loop) and uses
        DDPM seed ``seed + i``."""
        if not 0 < steps <= MAX_ROLLOUT_STEPS:
            raise ValueError(f"steps must be from 1 through {MAX_ROLLOUT_STEPS}")
        if diffusion_steps <= 0:
            raise ValueError("diffusion_steps must be positive")
        noise_rng = np.random.default_rng(seed)
        log = np.zeros(steps, np.int64)
        misses = 0
        self.policy.reset()
        began = self.clock()
        count = 0
        try:
            self.robot.reset()
            while count < steps:
                t0 = self.clock()
                condition = self.encode(self.robot.observe())
                noise_rng.standard_normal(self._noise.shape, dtype=np.float32, out=self._noise)
                self.policy.select_action_into(condition, self._noise, self._action, steps=diffusion_steps,
                                               scheduler=scheduler, seed=seed + count)
                if self.sync is not None:
                    self.sync()
                took = self.clock() - t0
                late = self._late(took)
                misses += int(late)
                self._dispatch(late, took)
                log[count] = took
                count += 1
        finally:
            self.robot.stop()
        return LoopReport(latencies_ns=log[:count], missed_deadlines=misses, on_miss=self.on_miss.value,
                          elapsed_ms=(self.clock() - began) / 1e6)


def run_rollout(policy: DiffusionPolicy, robot: Robot, encode_condition: Callable[[np.ndarray], np.ndarray], *,
                steps: int, seed: int = 0, diffusion_steps: int = 10, scheduler: str = "ddim",
                period_ms: float | None = None, on_miss: str = "hold", sync: Callable[[], None] | None = None,
                clock_ns: Callable[[], int] = perf_counter_ns) -> LoopReport:
    """One bounded rollout through a ``ControlLoop`` (the `--on-miss` entry point)."""
    loop = ControlLoop(policy, robot, encode_condition, period_ms=period_ms, on_miss=on_miss, sync=sync,
                       clock_ns=clock_ns)
    return loop.run(steps, seed=seed, diffusion_steps=diffusion_steps, scheduler=scheduler)
