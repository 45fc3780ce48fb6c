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
    assert device_malloc_count() == before
    e.close()
