"""The allocation-free flow entry point (fe_engine_sample_condition_static).

It exists for callers that cannot call cudaMalloc while they sample (a
fixed-period control loop, where cudaMalloc may block and synchronise the
device, or a host process whose device memory another runtime's pool
allocator claimed at start-up): its scratch is a fixed
static device array instead of the engine's workspace.  This file checks,
through the C ABI, that two calls in a row match the existing device entry
point (fe_engine_sample_condition_device) within the flow tolerance of the
other tests, that no device allocation happens, and that an oversized request
is rejected.  It is named to be collected last and must pass alone in a fresh
process as well as after the other tests.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from flowedge_b200 import Engine
from flowedge_b200.engine import device_malloc_count

pytestmark = pytest.mark.gpu

GOLD = "tests/golden/mamba_flow_tiny.safetensors"


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def test_static_scratch_flow_matches_device_entry_point(golden):
    _, _, g = golden("mamba_flow_tiny")
    batch, steps = 3, 10
    rng = np.random.default_rng(5)
    cond = torch.from_numpy(rng.standard_normal((batch, g["cond"].shape[1]), dtype=np.float32)).cuda()
    noise = torch.from_numpy(rng.standard_normal((batch, g["noise"].shape[1]), dtype=np.float32)).cuda()
    e = Engine(GOLD, threads=0, device=0, precision="fp32", max_batch=batch)
    lib = e.lib
    stream = torch.cuda.Stream()
    for method in (0, 2):  # Euler, RK4
        expected = torch.empty_like(noise)
        assert lib.fe_engine_sample_condition_device(e.handle, _ptr(cond), _ptr(noise), batch, steps, method,
                                                     _ptr(expected), C.c_void_p(stream.cuda_stream)) == 0
        stream.synchronize()
        before = device_malloc_count()
        for _ in range(2):  # two calls in a row share (and reuse) the static array
            got = torch.full_like(noise, float("nan"))
            rc = lib.fe_engine_sample_condition_static(e.handle, _ptr(cond), _ptr(noise), batch, steps, method,
                                                       _ptr(got), C.c_void_p(stream.cuda_stream))
            assert rc == 0, lib.fe_engine_last_error()
            stream.synchronize()
            np.testing.assert_allclose(got.cpu().numpy(), expected.cpu().numpy(), atol=2e-5, rtol=1e-4)
        assert device_malloc_count() == before
    # the same solve for one row matches the reference's own golden output
    one = torch.empty((1, noise.shape[1]), dtype=torch.float32, device="cuda")
    c0 = torch.from_numpy(g["cond"][:1].copy()).cuda()
    n0 = torch.from_numpy(g["noise"][:1].copy()).cuda()
    assert lib.fe_engine_sample_condition_static(e.handle, _ptr(c0), _ptr(n0), 1, 10, 0, _ptr(one),
                                                 C.c_void_p(stream.cuda_stream)) == 0
    stream.synchronize()
    np.testing.assert_allclose(one.cpu().numpy()[0], g["euler_10"][0], atol=2e-5, rtol=1e-4)
    e.close()


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_static_scratch_runs_past_the_reserved_capacity(precision):
    """An engine reserved for one row serves 17 rows (the 16-row tile plus a
    ragged one) from the static array without allocating, and matches the
    device entry point after that entry point's workspace was grown to 17."""
    batch, steps = 17, 6
    rng = np.random.default_rng(17)
    e = Engine(GOLD, threads=0, device=0, precision=precision, max_batch=1)
    lib = e.lib
    cond = torch.from_numpy(rng.standard_normal((batch, 16), dtype=np.float32)).cuda()
    noise = torch.from_numpy(rng.standard_normal((batch, 6), dtype=np.float32)).cuda()
    stream = torch.cuda.Stream()
    got = []
    before = device_malloc_count()
    for _ in range(2):
        out = torch.full_like(noise, float("nan"))
        rc = lib.fe_engine_sample_condition_static(e.handle, _ptr(cond), _ptr(noise), batch, steps, 2, _ptr(out),
                                                   C.c_void_p(stream.cuda_stream))
        assert rc == 0, lib.fe_engine_last_error()
        stream.synchronize()
        got.append(out.cpu().numpy())
    assert device_malloc_count() == before
    e.reserve_batch(batch)
    expected = torch.empty_like(noise)
    assert lib.fe_engine_sample_condition_device(e.handle, _ptr(cond), _ptr(noise), batch, steps, 2, _ptr(expected),
                                                 C.c_void_p(stream.cuda_stream)) == 0
    stream.synchronize()
    for g in got:
        np.testing.assert_allclose(g, expected.cpu().numpy(), atol=2e-5, rtol=1e-4)
    e.close()


def test_static_scratch_rejects_oversized_requests():
    e = Engine(GOLD, threads=0, device=0, precision="fp32")
    big = 1 << 16  # rows whose scratch cannot fit the 4 MiB array
    cond = torch.zeros((big, 16), dtype=torch.float32, device="cuda")
    noise = torch.zeros((big, 6), dtype=torch.float32, device="cuda")
    out = torch.zeros_like(noise)
    before = device_malloc_count()
    rc = e.lib.fe_engine_sample_condition_static(e.handle, _ptr(cond), _ptr(noise), big, 4, 0, _ptr(out), None)
    assert rc == 2
    assert b"static array" in e.lib.fe_engine_last_error()
    # a row count whose scratch size would wrap around size_t is rejected the
    # same way, before any launch (the buffers are never read)
    huge = (1 << 64) // 8 - 1
    rc = e.lib.fe_engine_sample_condition_static(e.handle, _ptr(cond), _ptr(noise), huge, 4, 0, _ptr(out), None)
    assert rc == 2
    assert b"static array" in e.lib.fe_engine_last_error()
    assert device_malloc_count() == before
    # the engine's current device is left as the caller had it, and a valid
    # call after the rejections succeeds (no stale error is reported)
    assert torch.cuda.current_device() == 0
    rc = e.lib.fe_engine_sample_condition_static(e.handle, _ptr(cond), _ptr(noise), 2, 4, 0, _ptr(out), None)
    assert rc == 0, e.lib.fe_engine_last_error()
    e.synchronize()
    e.close()
