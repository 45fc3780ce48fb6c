"""End-to-end parity of the CUDA path (through the C ABI) with the reference.

* golden fixtures (tests/golden/): the reference's own outputs on its own
  converted checkpoints - fp32 mode must match within 1e-4..1e-3;
* the compiled reference core (oracle/_ref) on a PushT-shaped checkpoint
  (PushT U-Net) - DDIM-10 actions within max-abs 1e-3 (fp32);
* bf16 mode (this build's added precision) within max-abs 2e-2 of the fp32
  reference, as the north star sets for bf16 weights with fp32 accumulation.
"""

import numpy as np
import pytest

from flowedge_b200 import Engine
from flowedge_b200 import checkpoint as ck
from flowedge_b200.engine import device_malloc_count
from oracle import restate

pytestmark = pytest.mark.gpu

GOLD = "tests/golden"


def _engine(name, **kw):
    return Engine(f"{GOLD}/{name}.safetensors", threads=0, device=0, **kw)


@pytest.mark.parametrize("name", ["unet_tiny", "unet_small"])
def test_unet_golden_fp32(golden, name):
    _, _, g = golden(name)
    e = _engine(name, precision="fp32")
    assert e.model_metadata["model_digest"] == bytes(g["digest"])
    for i, ts in enumerate(g["timesteps"]):
        np.testing.assert_allclose(e.diffusion_denoise(g["cond"][0], g["noise"][0], float(ts)), g["eps"][i],
                                   atol=1e-4, rtol=1e-4)
    for steps in (1, 5, 10):
        for i in range(3):
            out = e.sample_diffusion(g["cond"][i], g["noise"][i], steps, "ddim")
            np.testing.assert_allclose(out, g[f"ddim_{steps}"][i], atol=1e-4, rtol=1e-4)
    for i in range(3):
        out = e.sample_diffusion(g["cond"][i], g["noise"][i], 5, "ddpm", seed=int(g["ddpm_seeds"][i]))
        np.testing.assert_allclose(out, g["ddpm_5"][i], atol=5e-4, rtol=5e-4)
    e.close()


@pytest.mark.parametrize("name", ["unet_tiny", "unet_small"])
def test_unet_golden_bf16(golden, name):
    _, _, g = golden(name)
    e = _engine(name, precision="bf16")
    for i in range(3):
        out = e.sample_diffusion(g["cond"][i], g["noise"][i], 10, "ddim")
        np.testing.assert_allclose(out, g["ddim_10"][i], atol=2e-2 * 4.0)  # action range up to 4 (unnormalised)
    e.close()


def test_unet_batched_matches_single_and_is_deterministic(golden):
    _, _, g = golden("unet_small")
    e = _engine("unet_small", precision="fp32", max_batch=3)
    batch = e.sample_diffusion_batch(g["cond"], g["noise"], 10, "ddim")
    np.testing.assert_allclose(batch, g["ddim_10"], atol=1e-4, rtol=1e-4)
    again = e.sample_diffusion_batch(g["cond"], g["noise"], 10, "ddim")
    np.testing.assert_array_equal(batch, again)
    ddpm = e.sample_diffusion_batch(g["cond"], g["noise"], 5, "ddpm", seed=42)
    np.testing.assert_allclose(ddpm, g["ddpm_5"], atol=5e-4, rtol=5e-4)  # sample b uses seed 42 + b
    e.close()


def test_no_allocation_after_warmup(golden):
    _, _, g = golden("unet_small")
    e = _engine("unet_small", precision="fp32", max_batch=3)
    e.sample_diffusion_batch(g["cond"], g["noise"], 10, "ddim")
    e.sample_diffusion(g["cond"][0], g["noise"][0], 10, "ddpm", seed=1)
    before = device_malloc_count()
    for _ in range(3):
        e.sample_diffusion_batch(g["cond"], g["noise"], 10, "ddim")
        e.sample_diffusion(g["cond"][0], g["noise"][0], 10, "ddpm", seed=1)
    assert device_malloc_count() == before
    e.close()


def test_unet_metadata_and_errors(golden):
    e = _engine("unet_tiny", precision="fp32")
    md = e.diffusion_metadata
    assert md["action_dim"] == 2 and md["horizon"] == 8 and md["train_timesteps"] == 20
    assert e.cuda_resident and e.action_horizon == 8 and e.condition_dim == 6
    with pytest.raises(RuntimeError, match="status 1"):
        e.sample_diffusion(np.zeros(6), np.zeros((8, 2)), 21)
    with pytest.raises(RuntimeError, match="status 5"):
        e.lib.fe_engine_sample_diffusion and e._check(
            e.lib.fe_engine_sample_diffusion(e.handle, np.zeros(6, np.float32).ctypes.data_as(
                __import__("ctypes").POINTER(__import__("ctypes").c_float)),
                np.zeros(16, np.float32).ctypes.data_as(__import__("ctypes").POINTER(__import__("ctypes").c_float)),
                10, 7, 0, np.zeros(16, np.float32).ctypes.data_as(
                    __import__("ctypes").POINTER(__import__("ctypes").c_float))))
    with pytest.raises(RuntimeError, match="status 4"):
        e.sample_condition(np.zeros(6), np.zeros(2))
    e.close()


@pytest.mark.parametrize("name", ["mamba_flow_tiny", "mamba_flow_bf16"])
def test_mamba_flow_golden(golden, name):
    _, _, g = golden(name)
    e = _engine(name, precision="fp32")
    assert e.model_metadata["model_digest"] == bytes(g["digest"])
    np.testing.assert_allclose(e.run(g["tokens"]), g["hidden"], atol=2e-5, rtol=1e-4)
    for solver, steps in (("euler", 10), ("heun", 3), ("rk4", 4)):
        for i in range(2):
            out = e.sample_condition(g["cond"][i], g["noise"][i], steps=steps, method=solver)
            np.testing.assert_allclose(out, g[f"{solver}_{steps}"][i], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(e.sample(g["tokens"], g["noise"][0], 10, "euler"), g["pipeline_euler_10"],
                               atol=2e-5, rtol=1e-4)
    e.reset()
    for i, tok in enumerate(g["tokens"][:5]):
        np.testing.assert_allclose(e.step(tok), g["decoded"][i], atol=2e-5, rtol=1e-4)
    snap = e.decode_state()
    # header up to the payload checksum is identical; the checksum covers
    # payload bytes that agree only to float tolerance
    assert snap[:88] == bytes(g["snapshot"][:88])
    np.testing.assert_allclose(np.frombuffer(snap[96:], np.float32), g["snapshot"][96:].view(np.float32),
                               atol=2e-5, rtol=1e-4)
    e.close()


def test_flow_resumable_and_cancel(golden):
    _, _, g = golden("mamba_flow_tiny")
    e = _engine("mamba_flow_tiny", precision="fp32")
    out = np.empty(6, np.float32)
    e.flow_begin(g["cond"][0], g["noise"][0], steps=10, method="euler")
    remaining = 10
    while remaining:
        remaining = e.flow_advance(out, step_budget=3)
    np.testing.assert_allclose(out, g["euler_10"][0], atol=2e-5, rtol=1e-4)
    assert e.flow_metadata["status"] == 1  # FE_ACTION_COMPLETE
    e.flow_begin(g["cond"][0], g["noise"][0], steps=10, method="euler", generation=5)
    e.flow_advance(out, step_budget=2)
    e.cancel_before(6)
    with pytest.raises(RuntimeError, match="status 8"):
        e.flow_advance(out, step_budget=2)
    assert e.flow_metadata["status"] == 2  # FE_ACTION_CANCELLED
    e.close()


def test_decode_snapshot_round_trip(golden):
    _, _, g = golden("mamba_flow_tiny")
    e = _engine("mamba_flow_tiny", precision="fp32")
    e.reset()
    for tok in g["tokens"][:3]:
        e.step(tok)
    snap = e.decode_state()
    a = e.step(g["tokens"][3])
    e.restore_decode_state(snap)
    b = e.step(g["tokens"][3])
    np.testing.assert_array_equal(a, b)
    corrupt = bytearray(snap)
    corrupt[100] ^= 0xFF
    with pytest.raises(RuntimeError, match="status 10"):
        e.restore_decode_state(bytes(corrupt))
    e.close()


def _reference_run(path, cond, noise, steps=10, eps_t=None):
    from oracle import reference

    ref = reference.ReferenceEngine(path, threads=8)
    out = np.stack([ref.sample_diffusion(cond[i], noise[i], steps) for i in range(cond.shape[0])])
    eps = ref.diffusion_denoise(cond[0], noise[0], eps_t) if eps_t is not None else None
    ref.close()
    return out, eps


def _needs_reference():
    from oracle import reference

    if not reference.available():
        pytest.skip("oracle/_ref not built")


def test_pusht_fp32_ddim10_matches_reference_core(tmp_path):
    """PushT U-Net (fp32, batch 1) at full size against the
    compiled reference core: epsilon within 1e-4, DDIM-10 actions within 1e-3."""
    _needs_reference()
    tensors, meta = ck.diffusion_tensors(ck.PUSHT, seed=0)
    path = tmp_path / "pusht.safetensors"
    ck.write_checkpoint(path, tensors, metadata=meta)
    rng = np.random.default_rng(0)
    cond = rng.standard_normal((2, 132)).astype(np.float32)
    noise = rng.standard_normal((2, 16, 2)).astype(np.float32)
    expected, eps_ref = _reference_run(path, cond, noise, eps_t=90.0)
    e = Engine(path, threads=0, device=0, precision="fp32", max_batch=2)
    np.testing.assert_allclose(e.diffusion_denoise(cond[0], noise[0], 90.0), eps_ref, atol=1e-4, rtol=1e-4)
    out = np.stack([e.sample_diffusion(cond[i], noise[i], 10) for i in range(2)])
    err = float(np.abs(out - expected).max())
    print(f"PushT fp32 DDIM-10 max-abs vs reference: {err:.3g}")
    assert err <= 1e-3
    e.close()


def test_pusht_bf16_paths_match_reference_on_same_weights(tmp_path):
    """bf16 mode on bf16-representable weights, against the reference core run
    on the very same weights (stored as fp32, which the reference accepts).

    * batch-1 program (fp16 hi/lo activations on mma.sync): max-abs <= 1e-3
    * weight-streaming path (batch 2, fp32 activations): max-abs <= 1e-3
    * tensor-core path (batch 32, bf16 activations, fp32 accumulate): <= 2e-2
    and, for the record, the quantisation error of bf16 weights against the
    fp32-weight model (printed; DDIM amplifies epsilon errors by up to
    1/sqrt(alpha_bar) ~ 6 at the first steps)."""
    _needs_reference()
    tensors, meta = ck.diffusion_tensors(ck.PUSHT, seed=0)
    rounded = {k: (ck.bf16_bits_to_f32(ck.to_bf16_bits(v)) if v.ndim >= 2 else v) for k, v in tensors.items()}
    path = tmp_path / "pusht_bf16w.safetensors"
    ck.write_checkpoint(path, rounded, metadata=meta)
    rng = np.random.default_rng(1)
    cond = rng.standard_normal((32, 132)).astype(np.float32)
    noise = rng.standard_normal((32, 16, 2)).astype(np.float32)
    expected, _ = _reference_run(path, cond, noise)
    e = Engine(path, threads=0, device=0, precision="bf16", max_batch=32)
    single = e.sample_diffusion(cond[0], noise[0], 10)  # batch 1: the persistent small-batch program
    err_single = float(np.abs(single - expected[0]).max())
    small = e.sample_diffusion_batch(cond[:2], noise[:2], 10)
    err_small = float(np.abs(small - expected[:2]).max())
    big = e.sample_diffusion_batch(cond, noise, 10)
    err_big = float(np.abs(big - expected).max())
    e.close()
    print(f"PushT bf16 weights: batch-1 program max-abs {err_single:.3g}, streaming path max-abs {err_small:.3g}, "
          f"tensor path max-abs {err_big:.3g}")
    assert err_single <= 1e-3
    assert err_small <= 1e-3
    assert err_big <= 2e-2


def test_bimanual_c4_bf16_tensor_path_matches_reference_on_same_weights(tmp_path):
    """The bench's bimanual U-Net (A14, H64, dims
    512/1024/2048, 8 groups) in bf16 mode, on bf16-representable weights,
    against the reference core on the same weights: DDIM-10 actions within
    max-abs 2e-2.  Batch 8 x horizon 64 takes the tensor path, where every
    GroupNorm is applied in the conv epilogues: groups of 64 and 128 channels
    in 128-row tiles, the 256-channel groups of the 2048-channel stage in
    256-row tiles."""
    _needs_reference()
    from oracle import reference

    tensors, meta = ck.diffusion_tensors(ck.BIMANUAL, seed=3)
    path = tmp_path / "bimanual_bf16w.safetensors"
    ck.write_checkpoint(path, _round_bf16(tensors), metadata=meta)
    rng = np.random.default_rng(4)
    cond = rng.standard_normal((8, 284)).astype(np.float32)
    noise = rng.standard_normal((8, 64, 14)).astype(np.float32)
    ref = reference.ReferenceEngine(path, threads=8)
    expected = np.stack([ref.sample_diffusion(cond[i], noise[i], 10) for i in range(8)])
    ref.close()
    e = Engine(path, threads=0, device=0, precision="bf16", max_batch=8)
    got = e.sample_diffusion_batch(cond, noise, 10)
    e.close()
    err = float(np.abs(got - expected).max())
    print(f"C4 bimanual bf16 tensor path DDIM-10 max-abs vs reference: {err:.3g}")
    assert err <= 2e-2


def _round_bf16(tensors):
    return {k: (ck.bf16_bits_to_f32(ck.to_bf16_bits(v)) if v.ndim >= 2 and "embeddings" not in k
                and not k.endswith("A_log") else v) for k, v in tensors.items()}


def test_flow_c2_fp32_matches_reference_core(tmp_path):
    """Flow head (350 / 1024 x 3 / cond 512), fp32, batch 1:
    Euler-10 and RK4-4 against the compiled reference core (bar 1e-3)."""
    _needs_reference()
    from oracle import reference

    path = tmp_path / "flow_c2.safetensors"
    ck.write_checkpoint(path, ck.flow_tensors(ck.FLOW_C2, seed=2))
    rng = np.random.default_rng(2)
    cond = rng.standard_normal(512).astype(np.float32)
    x0 = rng.standard_normal(350).astype(np.float32)
    ref = reference.ReferenceEngine(path, threads=8)
    e = Engine(path, threads=0, device=0, precision="fp32")
    for solver, steps in (("euler", 10), ("rk4", 4), ("heun", 5)):
        expected = ref.sample_condition(cond, x0, steps, solver)
        got = e.sample_condition(cond, x0, steps=steps, method=solver)
        err = float(np.abs(got - expected).max())
        print(f"C2 flow fp32 {solver}-{steps} max-abs vs reference: {err:.3g}")
        assert err <= 1e-3
    ref.close()
    e.close()


def test_flow_c2_bf16_batched_tensor_path(tmp_path):
    """C2 at batch 256 in bf16 mode (the persistent tcgen05 solve: fp16
    operands, the ODE stage in the output projection's epilogue) against the
    restatement on the same bf16-rounded weights (bar 2e-2), for each solver
    and for a ragged batch of 300 rows."""
    tensors = _round_bf16(ck.flow_tensors(ck.FLOW_C2, seed=3))
    path = tmp_path / "flow_c2_bf16w.safetensors"
    ck.write_checkpoint(path, tensors)
    rng = np.random.default_rng(3)
    cond = rng.standard_normal((256, 512)).astype(np.float32)
    x0 = rng.standard_normal((256, 350)).astype(np.float32)
    flow = restate.FlowModel(tensors)
    e = Engine(path, threads=0, device=0, precision="bf16", max_batch=300)
    for solver, steps in (("euler", 10), ("rk4", 4), ("heun", 3)):
        got = e.sample_condition_batch(cond, x0, steps=steps, method=solver)
        expected = flow.sample(cond, x0, steps, solver)
        err = float(np.abs(got - expected).max())
        print(f"C2 flow bf16 batch-256 {solver}-{steps} max-abs vs restatement: {err:.3g}")
        assert err <= 2e-2
    # a ragged token block (300 rows: one full 256-row block and 44 rows)
    cond3 = rng.standard_normal((300, 512)).astype(np.float32)
    x3 = rng.standard_normal((300, 350)).astype(np.float32)
    got3 = e.sample_condition_batch(cond3, x3, steps=5, method="euler")
    err3 = float(np.abs(got3 - flow.sample(cond3, x3, 5, "euler")).max())
    print(f"C2 flow bf16 batch-300 euler-5 max-abs vs restatement: {err3:.3g}")
    assert err3 <= 2e-2
    # the small-batch (weight-streaming) path on the same engine
    got1 = e.sample_condition(cond[0], x0[0], steps=10, method="euler")
    assert np.abs(got1 - flow.sample(cond[:1], x0[:1], 10, "euler")[0]).max() <= 1e-3
    e.close()


def test_flow_c2_fp32_batched_split_tensor_path(tmp_path):
    """C2 at batch 256 in fp32 mode: tcgen05 GEMMs over fp16 hi / lo splits of
    weights and activations, against the fp32 restatement (bar 1e-3), and a
    batch-1 call (CUDA-core fp32 path) against the same rows."""
    tensors = ck.flow_tensors(ck.FLOW_C2, seed=4)
    path = tmp_path / "flow_c2_fp32.safetensors"
    ck.write_checkpoint(path, tensors)
    rng = np.random.default_rng(4)
    cond = rng.standard_normal((256, 512)).astype(np.float32)
    x0 = rng.standard_normal((256, 350)).astype(np.float32)
    flow = restate.FlowModel(tensors)
    e = Engine(path, threads=0, device=0, precision="fp32", max_batch=256)
    for solver, steps in (("euler", 10), ("rk4", 4), ("heun", 3)):
        got = e.sample_condition_batch(cond, x0, steps=steps, method=solver)
        expected = flow.sample(cond, x0, steps, solver)
        err = float(np.abs(got - expected).max())
        print(f"C2 flow fp32 batch-256 {solver}-{steps} max-abs vs restatement: {err:.3g}")
        assert err <= 1e-3
    got1 = e.sample_condition(cond[5], x0[5], steps=10, method="euler")
    batch = e.sample_condition_batch(cond, x0, steps=10, method="euler")
    assert np.abs(got1 - batch[5]).max() <= 1e-3
    e.close()


def _mamba_flow_c3(seed):
    t = ck.mamba_tensors(ck.MAMBA_C3, seed=seed)
    t.update(ck.flow_tensors(ck.FLOW_C2, seed=seed + 1))
    return t


def test_mamba_c3_fp32_matches_reference_core(tmp_path):
    """Mamba 8 x 512 (di 1024, ds 16, L = 128) feeding the
    C2 flow head, fp32 batch 1, against the compiled reference core."""
    _needs_reference()
    from oracle import reference

    path = tmp_path / "mamba_c3.safetensors"
    ck.write_checkpoint(path, _mamba_flow_c3(4))
    tokens = np.arange(128, dtype=np.int32)
    rng = np.random.default_rng(4)
    x0 = rng.standard_normal(350).astype(np.float32)
    ref = reference.ReferenceEngine(path, threads=8)
    e = Engine(path, threads=0, device=0, precision="fp32")
    hidden = e.run(tokens)
    expected = ref.run(tokens, 512)
    err_h = float(np.abs(hidden - expected).max())
    act = e.sample(tokens, x0, 10, "euler")
    err_a = float(np.abs(act - ref.sample(tokens, x0, 10, "euler")).max())
    print(f"C3 Mamba fp32 hidden max-abs {err_h:.3g}, Mamba->flow Euler-10 action max-abs {err_a:.3g}")
    assert err_h <= 1e-3 and err_a <= 1e-3
    ref.close()
    e.close()


def test_mamba_c3_bf16_batched_tensor_path(tmp_path):
    """C3 at batch 4 x 128 tokens in bf16 mode (tcgen05 projections) against the
    restatement on the same bf16-rounded weights."""
    tensors = _round_bf16(_mamba_flow_c3(5))
    path = tmp_path / "mamba_c3_bf16w.safetensors"
    ck.write_checkpoint(path, tensors)
    rng = np.random.default_rng(5)
    tokens = rng.integers(0, 128, size=(4, 128)).astype(np.int32)
    model = restate.MambaModel(tensors)
    e = Engine(path, threads=0, device=0, precision="bf16", max_batch=4)
    hidden = e.run_batch(tokens)
    expected = np.stack([model.run(tokens[i]) for i in range(4)])
    err = float(np.abs(hidden - expected).max())
    print(f"C3 Mamba bf16 batch-4 hidden max-abs vs restatement: {err:.3g}")
    assert err <= 2e-2
    x0 = rng.standard_normal((4, 350)).astype(np.float32)
    act = e.sample_batch(tokens, x0, 10, "euler")
    flow = restate.FlowModel(tensors)
    expected_act = np.stack([flow.sample(expected[i, -1], x0[i], 10, "euler") for i in range(4)])
    assert np.abs(act - expected_act).max() <= 2e-2
    e.close()


def test_mamba_c3_fp32_split_tensor_path_matches_cuda_cores(tmp_path):
    """fp32 Mamba projections on the tensor cores (fp16 hi/lo split, from 128
    tokens) against the same engine's CUDA-core fp32 path (below 128 tokens),
    fp32 tolerance 1e-3."""
    tensors = _mamba_flow_c3(6)
    path = tmp_path / "mamba_c3_split.safetensors"
    ck.write_checkpoint(path, tensors)
    rng = np.random.default_rng(6)
    tokens = rng.integers(0, 128, size=(3, 64)).astype(np.int32)
    e = Engine(path, threads=0, device=0, precision="fp32", max_batch=3)
    batched = e.run_batch(tokens)  # 192 tokens: tensor-core split path
    single = np.stack([e.run(tokens[i]) for i in range(3)])  # 64 tokens: CUDA cores
    err = float(np.abs(batched - single).max())
    print(f"C3 Mamba fp32 split tensor path vs CUDA cores max-abs {err:.3g}")
    assert err <= 1e-3
    e.close()
