"""One rank of the two-process gloo check of the batch-sharded path
(tests/test_shard_gloo.py): RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT
come from the environment, the output file from argv[1].

Each rank samples its contiguous shard with the batched engine's seeding
(sample j of a call with seed s draws from seed s + j), the numpy oracle
standing in for the rank's GPU engine, then gathers every rank's actions and
the maximum of a per-rank time with the helpers that bench.py uses.
"""

import datetime
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))

from flowedge_b200 import checkpoint as ck  # noqa: E402
from flowedge_b200.shard import gather_rows, max_over_ranks, shard_range, shard_seed  # noqa: E402
from oracle import restate  # noqa: E402

SPEC = ck.DiffusionSpec(action_dim=2, horizon=8, condition_dim=12, down_dims=(16, 32, 64), timestep_dim=16,
                        train_timesteps=20)
BATCH, STEPS, SEED = 4, 3, 77


def inputs():
    rng = np.random.default_rng(11)
    cond = rng.standard_normal((BATCH, SPEC.condition_dim), dtype=np.float32)
    noise = rng.standard_normal((BATCH, SPEC.horizon, SPEC.action_dim), dtype=np.float32)
    return cond, noise


def sample_shard(model, cond, noise, world, rank):
    offset, size = shard_range(BATCH, world, rank)
    seed = shard_seed(SEED, offset)
    return np.stack([model.sample(cond[offset + j], noise[offset + j], STEPS, "ddpm", seed=seed + j)
                     for j in range(size)])


def main(out_path):
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    world, rank = dist.get_world_size(), dist.get_rank()
    tensors, _ = ck.diffusion_tensors(SPEC, seed=3)
    model = restate.DiffusionModel(tensors)
    cond, noise = inputs()
    local = sample_shard(model, cond, noise, world, rank)
    gathered = gather_rows(torch.from_numpy(local), dist).numpy()
    slowest = max_over_ranks(float(rank + 1), dist)
    if rank == 0:
        np.savez(out_path, gathered=gathered, slowest=slowest, world=world)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
