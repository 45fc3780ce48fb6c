"""Host logic of the batch-sharded multi-GPU path (flowedge_b200/shard.py),
on CPU: shard bounds, shard-invariant DDPM seeds, and the gather / max-over-
ranks collectives with two gloo ranks on 127.0.0.1."""

import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from flowedge_b200.shard import shard_range, shard_seed

HERE = Path(__file__).resolve().parent


@pytest.mark.parametrize("batch,world", [(4096, 1), (4096, 2), (4096, 8), (5, 2), (3, 4), (0, 2)])
def test_shards_are_contiguous_balanced_and_cover_the_batch(batch, world):
    bounds = [shard_range(batch, world, r) for r in range(world)]
    start = 0
    for offset, size in bounds:
        assert offset == start
        start += size
    assert start == batch
    sizes = [s for _, s in bounds]
    assert max(sizes) - min(sizes) <= 1


def test_shard_seed_keeps_each_sample_on_its_global_seed():
    for world in (1, 2, 4, 8):
        for rank in range(world):
            offset, size = shard_range(64, world, rank)
            assert [shard_seed(5, offset) + j for j in range(size)] == [5 + offset + j for j in range(size)]


def test_invalid_shard_requests_are_rejected():
    for args in ((4, 0, 0), (4, 2, 2), (4, 2, -1), (-1, 2, 0)):
        with pytest.raises(ValueError):
            shard_range(*args)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_reproduce_the_single_process_batch(tmp_path):
    sys.path.insert(0, str(HERE))
    import shard_worker as w
    from oracle import restate
    from flowedge_b200 import checkpoint as ck

    out = tmp_path / "gathered.npz"
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()), WORLD_SIZE="2")
    procs = [subprocess.Popen([sys.executable, str(HERE / "shard_worker.py"), str(out)], env=dict(env, RANK=str(r)))
             for r in range(2)]
    try:
        codes = [p.wait(timeout=300) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert codes == [0, 0]
    got = np.load(out)
    assert int(got["world"]) == 2
    assert float(got["slowest"]) == 2.0  # max of the ranks' values 1 and 2

    tensors, _ = ck.diffusion_tensors(w.SPEC, seed=3)
    cond, noise = w.inputs()
    single = w.sample_shard(restate.DiffusionModel(tensors), cond, noise, 1, 0)
    # same arithmetic, same per-sample seeds: bitwise equal
    np.testing.assert_array_equal(got["gathered"], single)
