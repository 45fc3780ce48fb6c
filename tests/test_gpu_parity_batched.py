"""Parity of the batched kernels behind the bench's secondary lines, against the
compiled reference core (oracle/_ref) on sampled rows of the same inputs.

* Mamba (the 8 x 512 encoder: d_inner 1024, d_state 16, d_conv 4, dt_rank 32):
  - 64 sequences of 128 tokens reach the many-sequence selective scan
    (`scan_staged_kernel<16, 32, *>`, chosen when batch * d_inner >= 32768:
    eight 16-step tiles) at the bench's sequence length;
  - 640 sequences of 16 tokens also reach the register-window causal conv
    (`causal_conv_kernel`, chosen when batch * d_inner / 4 >= 1024 * SMs);
  - 2 sequences of 13 tokens reach the many-sequence scan at a small batch,
    because 13 steps do not split into the chunked scan's 8-step chunks (one
    ragged tile), and 3 sequences of 37 tokens run it over two whole tiles
    and a ragged third;
  - in bf16 mode the tensor-path in-projection takes the causal conv into its
    epilogue when the sequence length divides its 256-token blocks: 64 x 128
    and 640 x 16 run that way, 2 x 256 has a whole block per sequence (three
    of the four column slices of every tile continue a sequence begun in the
    slice before), and 4 x 37 (148 tokens: tensor path, 37 does not divide
    the block) keeps the separate conv kernel. With the conv fused the
    many-sequence scan stages u from its fp16 copy (64 x 128, 640 x 16, and
    600 x 8: one ragged 8-step tile).
  Each in fp32 mode (tensor cores on fp16 hi / lo splits, bar 1e-3) and in bf16
  mode on bf16-rounded weights (bar 2e-2), per-row against the reference's
  `Mamba::forward` (src/core/models/mamba/mamba.cc:232-315; scan at
  src/core/kernels/cpu/kernels_scalar.cc:133-169).
* PushT U-Net DDPM-5 on the tensor path (batch 32 x horizon 16 = 512 tokens,
  bf16 mode): the device-regenerated DDPM noise with per-sample seeds
  seed + b against the reference sampler (heads/diffusion/diffusion.cc:946-963)
  run on the same bf16-rounded weights, bar 2e-2.
"""

import numpy as np
import pytest

from flowedge_b200 import Engine
from flowedge_b200 import checkpoint as ck

pytestmark = pytest.mark.gpu


def _needs_reference():
    from oracle import reference

    if not reference.available():
        pytest.skip("oracle/_ref not built")


def _round_bf16(tensors):
    return {k: (ck.bf16_bits_to_f32(ck.to_bf16_bits(v)) if v.ndim >= 2 and "embeddings" not in k
                and not k.endswith("A_log") else v) for k, v in tensors.items()}


@pytest.fixture(scope="module")
def mamba_checkpoints(tmp_path_factory):
    root = tmp_path_factory.mktemp("mamba_batched")
    tensors = ck.mamba_tensors(ck.MAMBA_C3, seed=21)
    paths = {"fp32": root / "mamba_fp32.safetensors", "bf16": root / "mamba_bf16w.safetensors"}
    ck.write_checkpoint(paths["fp32"], tensors)
    ck.write_checkpoint(paths["bf16"], _round_bf16(tensors))
    return paths


CASES = [  # (batch, seq_len, rows compared with the reference)
    (64, 128, (0, 37, 63)),
    (640, 16, (0, 1, 318, 638, 639)),
    (2, 13, (0, 1)),
    (3, 37, (0, 2)),
    (2, 256, (0, 1)),
    (4, 37, (0, 3)),
    (600, 8, (0, 299, 599)),
]


@pytest.mark.parametrize("precision,bar", [("fp32", 1e-3), ("bf16", 2e-2)])
@pytest.mark.parametrize("batch,seq_len,rows", CASES, ids=[f"b{b}_L{l}" for b, l, _ in CASES])
def test_mamba_many_sequence_kernels_match_reference(mamba_checkpoints, precision, bar, batch, seq_len, rows):
    _needs_reference()
    from oracle import reference

    path = mamba_checkpoints[precision]
    rng = np.random.default_rng(batch * 1000 + seq_len)
    tokens = rng.integers(0, ck.MAMBA_C3.vocab, size=(batch, seq_len)).astype(np.int32)
    e = Engine(path, threads=0, device=0, precision=precision, max_batch=batch, max_sequence=seq_len)
    hidden = e.run_batch(tokens)
    e.close()
    assert np.isfinite(hidden).all()
    ref = reference.ReferenceEngine(path, threads=8)
    worst = 0.0
    for r in rows:
        expected = ref.run(tokens[r], ck.MAMBA_C3.d_model)
        worst = max(worst, float(np.abs(hidden[r] - expected).max()))
    ref.close()
    print(f"Mamba {precision} batch {batch} x {seq_len}: max-abs vs reference over rows {rows}: {worst:.3g}")
    assert worst <= bar


def test_pusht_ddpm_tensor_path_matches_reference_on_same_weights(tmp_path):
    _needs_reference()
    from oracle import reference

    tensors, meta = ck.diffusion_tensors(ck.PUSHT, seed=5)
    rounded = {k: (ck.bf16_bits_to_f32(ck.to_bf16_bits(v)) if v.ndim >= 2 else v) for k, v in tensors.items()}
    path = tmp_path / "pusht_bf16w.safetensors"
    ck.write_checkpoint(path, rounded, metadata=meta)
    rng = np.random.default_rng(6)
    batch, seed = 32, 11
    cond = rng.standard_normal((batch, 132)).astype(np.float32)
    noise = rng.standard_normal((batch, 16, 2)).astype(np.float32)
    e = Engine(path, threads=0, device=0, precision="bf16", max_batch=batch)
    got = e.sample_diffusion_batch(cond, noise, 5, "ddpm", seed=seed)
    again = e.sample_diffusion_batch(cond, noise, 5, "ddpm", seed=seed)
    other = e.sample_diffusion_batch(cond, noise, 5, "ddpm", seed=seed + 1000)
    e.close()
    np.testing.assert_array_equal(got, again)  # deterministic for a seed
    assert np.abs(got - other).max() > 1e-3  # and the seed reaches the noise
    ref = reference.ReferenceEngine(path, threads=8)
    rows = (0, 1, 7, 16, 30, 31)
    expected = np.stack([ref.sample_diffusion(cond[b], noise[b], 5, "ddpm", seed=seed + b) for b in rows])
    ref.close()
    err = float(np.abs(got[list(rows)] - expected).max())
    print(f"PushT bf16 tensor path DDPM-5 (batch {batch}) max-abs vs reference over rows {rows}: {err:.3g}")
    assert err <= 2e-2


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_load_rejects_weights_outside_the_fp16_storage_range(tmp_path, precision):
    """A conv weight beyond fp16's range (which both weight modes store in)
    fails the load with a message naming the tensor, instead of turning into
    inf on the device; the same model without it loads."""
    spec = ck.DiffusionSpec(action_dim=2, horizon=16, condition_dim=8, down_dims=(64, 128, 256), timestep_dim=32,
                            train_timesteps=20)
    tensors, meta = ck.diffusion_tensors(spec, seed=1)
    good = tmp_path / "good.safetensors"
    ck.write_checkpoint(good, tensors, metadata=meta)
    Engine(good, threads=0, device=0, precision=precision).close()
    bad_tensors = dict(tensors)
    w = bad_tensors["dp.m0.c1.w"].copy()
    w.flat[5] = 1.0e5
    bad_tensors["dp.m0.c1.w"] = w
    bad = tmp_path / "bad.safetensors"
    ck.write_checkpoint(bad, bad_tensors, metadata=meta)
    with pytest.raises(RuntimeError, match=r"dp\.m0\.c1\.w.*65504"):
        Engine(bad, threads=0, device=0, precision=precision)


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_reference_converted_file_recast_to_bf16_convs(tmp_path, golden, precision):
    """The golden U-Net fixture (written by the reference's converter, convs in
    F32) re-emitted with BF16 convs samples exactly like its fp32 twin (the same
    bf16-rounded convs stored as F32) in both precision modes, and the twin
    matches the reference core run on it; the batch reservation recorded in the
    file's metadata is what a device-buffer call of that batch needs."""
    import torch

    _needs_reference()
    from oracle import reference

    src = "tests/golden/unet_small.safetensors"
    bfc = tmp_path / "unet_small_bf16conv.safetensors"
    ck.recast_convs_bf16(src, bfc, max_batch=3)
    tensors, meta = ck.read_safetensors(src)
    twin_tensors = {k: (ck.bf16_bits_to_f32(ck.to_bf16_bits(v)) if v.ndim == 3 and k.startswith("dp.") else v)
                    for k, v in tensors.items()}
    twin = tmp_path / "unet_small_twin.safetensors"
    ck.write_safetensors(twin, twin_tensors, meta)
    _, _, g = golden("unet_small")
    cond, noise = g["cond"], g["noise"]
    e_bf = Engine(bfc, threads=0, device=0, precision=precision)  # reservation from the file's metadata
    e_tw = Engine(twin, threads=0, device=0, precision=precision)  # reservation 1
    d_cond, d_noise = torch.from_numpy(cond).cuda(), torch.from_numpy(noise).cuda()
    d_out = torch.empty_like(d_noise)
    e_bf.sample_diffusion_device(d_cond.data_ptr(), d_noise.data_ptr(), 3, d_out.data_ptr(), 10, "ddim")
    e_bf.synchronize()
    with pytest.raises(RuntimeError, match="status 2"):
        e_tw.sample_diffusion_device(d_cond.data_ptr(), d_noise.data_ptr(), 3, d_out.data_ptr(), 10, "ddim")
    a = e_bf.sample_diffusion_batch(cond, noise, 10, "ddim")
    b = e_tw.sample_diffusion_batch(cond, noise, 10, "ddim")
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(a, d_out.cpu().numpy())
    e_bf.close()
    e_tw.close()
    ref = reference.ReferenceEngine(twin, threads=8)
    expected = np.stack([ref.sample_diffusion(cond[i], noise[i], 10) for i in range(3)])
    ref.close()
    err = float(np.abs(a - expected).max())
    bar = 1e-4 if precision == "fp32" else 2e-2 * 4.0  # bf16 mode: action range up to 4 (unnormalised)
    print(f"recast BF16-conv file, {precision} mode: DDIM-10 max-abs vs reference on the twin {err:.3g}")
    assert err <= bar
