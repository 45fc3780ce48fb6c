#!/usr/bin/env python3
"""Regenerate the golden fixtures in this directory from the reference itself.

Run where the reference checkout and PyTorch are available, with
FLOWEDGE_REFERENCE naming the checkout:

    FLOWEDGE_REFERENCE=<path to FlowEdge> python tests/golden/make_golden.py [fixture names]

For each fixture it
  1. builds a small seeded model in the *source* layout the reference converter
     consumes (LeRobot ConditionalUnet1d from the reference's own
     tools/verification/verify_diffusion.py, or HF-Mamba + flow names),
  2. converts it with the reference's convert/convert.py,
  3. runs the reference core compiled by oracle/Makefile (oracle/_ref) on
     seeded inputs through its C ABI, and
  4. stores the converted checkpoint plus inputs/outputs as .safetensors/.npz.

The fixtures are the pins for both the numpy restatement (oracle/restate.py)
and this build's CUDA path.  Nothing at test time reads the reference checkout.
"""

from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch
from safetensors.torch import save_file

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if not os.environ.get("FLOWEDGE_REFERENCE"):
    sys.exit("set FLOWEDGE_REFERENCE to the reference FlowEdge checkout")
REF = Path(os.environ["FLOWEDGE_REFERENCE"])
sys.path.insert(0, str(REPO))

from oracle import reference as oracle_ref  # noqa: E402


def _reference_unet_module():
    spec = importlib.util.spec_from_file_location(
        "ref_verify_diffusion", REF / "tools" / "verification" / "verify_diffusion.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _convert(source_dir: Path, out: Path, arch: str, dtype: str = "f32"):
    subprocess.run([sys.executable, str(REF / "convert" / "convert.py"), str(source_dir), str(out),
                    "--arch", arch, "--dtype", dtype], check=True, stdout=subprocess.DEVNULL)


DIFFUSION_FIXTURES = {
    # name: (action_dim, horizon, condition_dim, down_dims, kernel, groups, temb, train_steps, seed)
    "unet_tiny": (2, 8, 6, [8, 16, 32], 5, 2, 8, 20, 3),
    "unet_small": (3, 16, 10, [16, 32, 64], 5, 8, 16, 100, 5),
}


def make_diffusion(name, params):
    a, h, c, dims, k, g, td, steps_t, seed = params
    verify = _reference_unet_module()
    torch.manual_seed(seed)
    model = verify.ConditionalUnet1d(a, c, dims, k, g, td).eval()
    with torch.no_grad():
        # Give GroupNorm affine parameters non-trivial values so the fixture
        # exercises them (PyTorch initialises them to 1 / 0).
        for module in model.modules():
            if isinstance(module, torch.nn.GroupNorm):
                module.weight.uniform_(0.5, 1.5)
                module.bias.uniform_(-0.3, 0.3)
    state = {f"diffusion.unet.{key}": value for key, value in model.state_dict().items()}
    action_min = torch.linspace(-2.0, 0.5, a)
    action_max = action_min + torch.linspace(1.0, 4.0, a)
    state["unnormalize_outputs.buffer_action.min"] = action_min
    state["unnormalize_outputs.buffer_action.max"] = action_max
    config = {
        "type": "diffusion", "beta_schedule": "squaredcos_cap_v2", "prediction_type": "epsilon",
        "use_film_scale_modulation": True, "use_group_norm": True,
        "normalization_mapping": {"ACTION": "MIN_MAX"}, "down_dims": dims,
        "output_features": {"action": {"shape": [a], "type": "ACTION"}},
        "horizon": h, "n_action_steps": 2, "n_obs_steps": 2, "kernel_size": k, "n_groups": g,
        "diffusion_step_embed_dim": td, "num_train_timesteps": steps_t, "clip_sample": True,
        "clip_sample_range": 1.0,
    }
    out_path = HERE / f"{name}.safetensors"
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        save_file(state, tmp / "model.safetensors")
        (tmp / "config.json").write_text(json.dumps(config))
        _convert(tmp, out_path, "diffusion")

    rng = np.random.default_rng(seed + 100)
    cond = rng.standard_normal((3, c)).astype(np.float32)
    noise = rng.standard_normal((3, h, a)).astype(np.float32)
    engine = oracle_ref.ReferenceEngine(out_path, threads=0)
    timesteps = np.array([0.0, 7.0, float(steps_t - 1)], np.float32)
    eps = np.stack([engine.diffusion_denoise(cond[0], noise[0], ts) for ts in timesteps])
    with torch.no_grad():
        eps_torch = np.stack([model(torch.from_numpy(noise[0][None]), torch.tensor([float(ts)]),
                                    torch.from_numpy(cond[0][None])).numpy()[0]
                              for ts in timesteps])
    ddim = {}
    for steps in (1, 5, 10):
        ddim[steps] = np.stack([engine.sample_diffusion(cond[i], noise[i], steps, "ddim")
                                for i in range(3)])
    ddpm = np.stack([engine.sample_diffusion(cond[i], noise[i], 5, "ddpm", seed=42 + i)
                     for i in range(3)])
    meta = engine.metadata()
    np.savez(HERE / f"{name}.npz", cond=cond, noise=noise, timesteps=timesteps, eps=eps,
             eps_torch=eps_torch, ddim_1=ddim[1], ddim_5=ddim[5], ddim_10=ddim[10], ddpm_5=ddpm,
             ddpm_seeds=np.array([42, 43, 44], np.uint64),
             digest=np.frombuffer(meta["digest"], np.uint8))
    engine.close()
    print(f"{name}: eps ref-vs-torch max-abs {np.abs(eps - eps_torch).max():.3g}")


MAMBA_FLOW_FIXTURES = {
    # name: (vocab, d_model, layers, d_inner, d_state, d_conv, dt_rank, action, hidden, mlp, time, dtype, seed)
    "mamba_flow_tiny": (20, 16, 2, 32, 4, 4, 4, 6, 32, 2, 8, "f32", 11),
    "mamba_flow_bf16": (24, 32, 2, 64, 8, 4, 4, 10, 64, 3, 16, "bf16", 13),
}


def _mamba_flow_state(params):
    vocab, dm, layers, di, ds, dc, dr, act, hid, mlp, td, _, seed = params
    gen = torch.Generator().manual_seed(seed)

    def u(*shape, fan_in):
        bound = fan_in ** -0.5
        return (torch.rand(*shape, generator=gen) * 2 - 1) * bound

    state = {"backbone.embedding.weight": torch.randn(vocab, dm, generator=gen)}
    for i in range(layers):
        p = f"backbone.layers.{i}."
        state[p + "norm.weight"] = 1 + 0.1 * torch.randn(dm, generator=gen)
        state[p + "mixer.in_proj.weight"] = u(2 * di, dm, fan_in=dm)
        state[p + "mixer.conv1d.weight"] = u(di, 1, dc, fan_in=dc)
        state[p + "mixer.conv1d.bias"] = u(di, fan_in=dc)
        state[p + "mixer.x_proj.weight"] = u(dr + 2 * ds, di, fan_in=di)
        state[p + "mixer.dt_proj.weight"] = u(di, dr, fan_in=dr)
        state[p + "mixer.dt_proj.bias"] = torch.log(torch.expm1(0.001 + 0.05 * torch.rand(di, generator=gen)))
        state[p + "mixer.A_log"] = torch.log(torch.arange(1, ds + 1, dtype=torch.float32)).repeat(di, 1)
        state[p + "mixer.D"] = torch.ones(di) + 0.1 * torch.randn(di, generator=gen)
        state[p + "mixer.out_proj.weight"] = u(dm, di, fan_in=di)
    state["backbone.norm_f.weight"] = 1 + 0.1 * torch.randn(dm, generator=gen)
    state["flow.in_proj.weight"] = u(hid, act, fan_in=act)
    state["flow.time_proj.weight"] = u(hid, td, fan_in=td)
    state["flow.cond_proj.weight"] = u(hid, dm, fan_in=dm)
    for i in range(mlp):
        state[f"flow.layers.{i}.weight"] = u(hid, hid, fan_in=hid)
    state["flow.out_proj.weight"] = u(act, hid, fan_in=hid)
    # an unrelated tensor the converter must drop
    state["lm_head.weight"] = torch.zeros(3, 3)
    return state


def make_mamba_flow(name, params):
    vocab, dm, layers, di, ds, dc, dr, act, hid, mlp, td, dtype, seed = params
    state = _mamba_flow_state(params)
    out_path = HERE / f"{name}.safetensors"
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp) / "model.safetensors"
        save_file(state, src)
        subprocess.run([sys.executable, str(REF / "convert" / "convert.py"), str(src), str(out_path),
                        "--arch", "mamba", "--dtype", dtype], check=True, stdout=subprocess.DEVNULL)
    rng = np.random.default_rng(seed + 100)
    tokens = rng.integers(0, vocab, size=9).astype(np.int32)
    cond = rng.standard_normal((2, dm)).astype(np.float32)
    noise = rng.standard_normal((2, act)).astype(np.float32)
    engine = oracle_ref.ReferenceEngine(out_path, threads=0)
    hidden = engine.run(tokens, dm)
    flows = {}
    for solver, steps in (("euler", 10), ("heun", 3), ("rk4", 4)):
        flows[solver] = np.stack([engine.sample_condition(cond[i], noise[i], steps, solver)
                                  for i in range(2)])
    pipeline = engine.sample(tokens, noise[0], 10, "euler")
    engine.reset()
    decoded = np.stack([engine.step(tok, dm) for tok in tokens[:5]])
    snapshot = np.frombuffer(engine.export_decode_state(), np.uint8)
    meta = engine.metadata()
    np.savez(HERE / f"{name}.npz", tokens=tokens, cond=cond, noise=noise, hidden=hidden,
             euler_10=flows["euler"], heun_3=flows["heun"], rk4_4=flows["rk4"],
             pipeline_euler_10=pipeline, decoded=decoded, snapshot=snapshot,
             digest=np.frombuffer(meta["digest"], np.uint8))
    engine.close()
    print(f"{name}: hidden norm {np.linalg.norm(hidden):.4f}")


# SmolVLA action expert at the shapes the reference loads (attention 960 = 15 x 64,
# K / V 320, MLP 2048).  The weights and the prefix cache are regenerated at test
# time from (spec, seed) by flowedge_b200.checkpoint, so the fixture holds only
# the inputs the generators do not make and the reference's outputs.
SMOLVLA_FIXTURES = {
    "smolvla_ref": dict(layers=4, chunk=10, prefix=24, masked=5, seed=11, timestep=0.7, steps=10),
    "smolvla_ref16": dict(layers=16, chunk=50, prefix=64, masked=9, seed=12, timestep=0.35, steps=10),
}


def make_smolvla(name, params):
    import dataclasses

    from flowedge_b200 import checkpoint as ck

    spec = dataclasses.replace(ck.SMOLVLA_REF, layers=params["layers"], chunk=params["chunk"],
                               prefix=params["prefix"])
    tensors = ck.smolvla_tensors(spec, params["seed"])
    keys, values, mask = ck.smolvla_prefix(spec, params["seed"] + 1, masked=params["masked"])
    rng = np.random.default_rng(params["seed"] + 2)
    noise = rng.standard_normal((spec.chunk, spec.action_dim), dtype=np.float32)
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / f"{name}.safetensors"
        ck.write_checkpoint(path, tensors, matrices="bf16")
        engine = oracle_ref.ReferenceEngine(path, threads=8)
        t = np.float32(params["timestep"])
        embed = engine.smolvla_embed_suffix(noise, t, spec.expert_width)
        hidden = engine.smolvla_run_expert(embed, keys, values, mask)
        project = engine.smolvla_project_actions(hidden, spec.action_dim)
        denoise = engine.smolvla_denoise(noise, t, keys, values, mask)
        sample = engine.smolvla_sample(noise, params["steps"], keys, values, mask)
        engine.close()
    np.savez(HERE / f"{name}.npz", noise=noise, timestep=t, embed=embed, hidden=hidden, project=project,
             denoise=denoise, sample=sample, params=np.array(json.dumps(params)))
    print(f"{name}: sample norm {np.linalg.norm(sample):.4f}")


def main():
    oracle_ref.build()
    only = sys.argv[1:]
    for name, params in DIFFUSION_FIXTURES.items():
        if not only or name in only:
            make_diffusion(name, params)
    for name, params in MAMBA_FLOW_FIXTURES.items():
        if not only or name in only:
            make_mamba_flow(name, params)
    for name, params in SMOLVLA_FIXTURES.items():
        if not only or name in only:
            make_smolvla(name, params)


if __name__ == "__main__":
    main()
