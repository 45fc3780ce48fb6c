"""Kernel-level numerics on the GPU: the tcgen05 GEMM and implicit-GEMM
convolution against a PyTorch fp32 reference of the same op on the same
bf16-rounded operands (fp32 accumulation in both; tolerance covers only the
summation order and the bf16 rounding of the conv output)."""

import ctypes as C

import numpy as np
import pytest
import torch

from flowedge_b200 import engine as fe
from flowedge_b200.checkpoint import bf16_bits_to_f32, to_bf16_bits

pytestmark = pytest.mark.gpu

u16p = C.POINTER(C.c_uint16)
f32p = C.POINTER(C.c_float)
f64p = C.POINTER(C.c_double)


@pytest.fixture(scope="module")
def lib():
    handle = fe.load_library()
    handle.febtest_gemm_16.argtypes = [u16p, C.c_int, C.c_int, u16p, C.c_int, f32p, C.c_int]
    handle.febtest_conv_16.argtypes = [u16p, C.c_int, C.c_int, C.c_int, u16p, f32p, C.c_int, C.c_int, C.c_int,
                                       f32p, f64p, C.c_int]
    return handle


def _to16(x, fp16):
    """float32 -> (16-bit raw bits, the exact float32 values they encode)."""
    if fp16:
        h = x.astype(np.float16)
        return h.view(np.uint16), h.astype(np.float32)
    bits = to_bf16_bits(x)
    return bits, bf16_bits_to_f32(bits)


@pytest.mark.parametrize("fp16", [0, 1])
@pytest.mark.parametrize("M,K,N", [(128, 64, 256), (384, 350, 300), (1024, 1024, 4096), (64, 32, 1)])
def test_tc_gemm_matches_torch(lib, M, K, N, fp16):
    rng = np.random.default_rng(M + K + N)
    a, af = _to16(rng.standard_normal((M, K), dtype=np.float32), fp16)
    b, bf = _to16(rng.standard_normal((N, K), dtype=np.float32), fp16)
    c = np.empty((N, M), np.float32)
    rc = lib.febtest_gemm_16(a.ctypes.data_as(u16p), M, K, b.ctypes.data_as(u16p), N, c.ctypes.data_as(f32p), fp16)
    assert rc == 0
    ref = (torch.from_numpy(bf).double() @ torch.from_numpy(af).double().T).numpy()
    np.testing.assert_allclose(c, ref, atol=1e-3 * np.sqrt(K), rtol=1e-4)


@pytest.mark.parametrize("fp16", [0, 1])
@pytest.mark.parametrize("B,L,C,OC,k,gch", [(4, 64, 64, 128, 5, 64), (16, 16, 128, 256, 5, 256),
                                              (64, 4, 256, 128, 5, 32), (3, 32, 64, 128, 1, 0)])
def test_tc_conv_matches_torch(lib, B, L, C, OC, k, gch, fp16):
    rng = np.random.default_rng(B * L + C)
    x, xf = _to16(rng.standard_normal((B, L, C), dtype=np.float32), fp16)
    w, wf = _to16((rng.standard_normal((OC, C, k), dtype=np.float32) / np.sqrt(C * k)).astype(np.float32), fp16)
    bias = rng.standard_normal(OC).astype(np.float32)
    y = np.empty((B, L, OC), np.float32)
    groups = OC // gch if gch else 0
    stats = np.zeros((B, max(groups, 1), 2), np.float64)
    rc = lib.febtest_conv_16(x.ctypes.data_as(u16p), B, L, C, w.ctypes.data_as(u16p),
                             bias.ctypes.data_as(f32p), OC, k, gch, y.ctypes.data_as(f32p),
                             stats.ctypes.data_as(f64p), fp16)
    assert rc == 0
    xt = torch.from_numpy(xf).double().permute(0, 2, 1)
    wt = torch.from_numpy(wf).double()
    ref = torch.nn.functional.conv1d(xt, wt, torch.from_numpy(bias).double(), padding=k // 2)
    ref = ref.permute(0, 2, 1).numpy()
    np.testing.assert_allclose(y, ref, atol=2e-2, rtol=1e-2 if not fp16 else 2e-3)  # y is stored in 16 bits
    if groups:
        g = ref.reshape(B, L, groups, gch)
        np.testing.assert_allclose(stats[..., 0], g.sum(axis=(1, 3)), rtol=1e-4, atol=1e-2)
        np.testing.assert_allclose(stats[..., 1], (g * g).sum(axis=(1, 3)), rtol=1e-4, atol=1e-2)
