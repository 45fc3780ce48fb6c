"""Synthetic checkpoints in FlowEdge's converted safetensors layout.

The reference converter (convert/convert.py) turns LeRobot / HF checkpoints
into the short tensor names the runtime loads: `dp.*` for the Diffusion Policy
U-Net (convert/convert.py:499-574, metadata vector at :475-492), `flow.*` for
the flow-matching head and `backbone.*` for Mamba (HF names,
src/core/models/mamba/mamba.cc:103-222).  Real checkpoints need the network,
so the benchmark and the GPU tests build random-init models directly in that
layout with PyTorch's default initialisation (Linear / Conv weights and biases
U(-1/sqrt(fan_in), 1/sqrt(fan_in)); GroupNorm weight 1, bias 0).  The same
arrays written through the reference converter produce an identical file
content (checked by the golden-fixture tests).

`convs="bf16"` stores the U-Net conv weights as BF16, and
`recast_convs_bf16` does the same to a file the reference converter wrote
(`python -m flowedge_b200.checkpoint recast-convs SRC DST [--max-batch N]`).
That is a new precision mode of this build: the reference loader accepts only
F32 convs (src/core/heads/diffusion/diffusion.cc:656-660) and the reference
converter casts only 2-D tensors (convert/convert.py:602-610).
"""

from __future__ import annotations

import hashlib
import json
import math
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

__all__ = [
    "DiffusionSpec",
    "FlowSpec",
    "MambaSpec",
    "diffusion_tensors",
    "flow_tensors",
    "mamba_tensors",
    "to_bf16_bits",
    "bf16_bits_to_f32",
    "write_safetensors",
    "read_safetensors",
    "PUSHT",
    "BIMANUAL",
    "FLOW_C2",
    "MAMBA_C3",
    "SmolVLASpec",
    "smolvla_tensors",
    "smolvla_prefix",
    "SMOLVLA_C5",
    "SMOLVLA_REF",
    "recast_convs_bf16",
]


# ----------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, as torch.Tensor.to(torch.bfloat16))


def to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    rounding = ((bits >> 16) & 1) + np.uint32(0x7FFF)
    out = ((bits + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(values)
    if nan.any():
        out[nan] = np.uint16(0x7FC0)
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------
# safetensors container (header: u64 little-endian length + JSON; raw data)


def write_safetensors(path, tensors: dict, metadata: dict | None = None) -> None:
    """Write `tensors` (name -> float32 ndarray, or ("BF16", uint16 ndarray))."""
    header: dict = {}
    blobs = []
    offset = 0
    for name, value in tensors.items():
        if isinstance(value, tuple):
            dtype, array = value
        else:
            dtype, array = "F32", np.ascontiguousarray(value, dtype=np.float32)
        array = np.ascontiguousarray(array)
        raw = array.tobytes()
        header[name] = {
            "dtype": dtype,
            "shape": list(array.shape),
            "data_offsets": [offset, offset + len(raw)],
        }
        blobs.append(raw)
        offset += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    encoded = json.dumps(header, separators=(",", ":")).encode("utf-8")
    encoded += b" " * ((8 - len(encoded) % 8) % 8)
    with open(path, "wb") as stream:
        stream.write(struct.pack("<Q", len(encoded)))
        stream.write(encoded)
        for raw in blobs:
            stream.write(raw)


def read_safetensors(path) -> tuple[dict, dict]:
    """Return ({name: float32 ndarray}, metadata). BF16 tensors are widened."""
    data = Path(path).read_bytes()
    (length,) = struct.unpack("<Q", data[:8])
    header = json.loads(data[8 : 8 + length])
    base = 8 + length
    metadata = header.pop("__metadata__", {})
    out = {}
    for name, entry in header.items():
        begin, end = entry["data_offsets"]
        raw = data[base + begin : base + end]
        if entry["dtype"] == "F32":
            array = np.frombuffer(raw, dtype=np.float32)
        elif entry["dtype"] == "BF16":
            array = bf16_bits_to_f32(np.frombuffer(raw, dtype=np.uint16))
        else:
            raise ValueError(f"unsupported dtype {entry['dtype']} for {name}")
        out[name] = array.reshape(entry["shape"]).copy()
    return out, metadata


# ----------------------------------------------------------------------------
# model specifications (the benchmarked workloads are module constants below)


@dataclass(frozen=True)
class DiffusionSpec:
    action_dim: int
    horizon: int
    condition_dim: int
    down_dims: tuple = (512, 1024, 2048)
    kernel: int = 5
    groups: int = 8
    timestep_dim: int = 128
    train_timesteps: int = 100
    action_steps: int = 8
    observation_steps: int = 2
    clip_sample: bool = True
    clip_sample_range: float = 1.0
    action_min: tuple | None = None
    action_max: tuple | None = None


@dataclass(frozen=True)
class FlowSpec:
    action_dim: int = 350
    hidden: int = 1024
    layers: int = 3
    time_dim: int = 128
    cond_dim: int = 512


@dataclass(frozen=True)
class MambaSpec:
    vocab: int = 128
    d_model: int = 512
    n_layers: int = 8
    d_inner: int = 1024
    d_state: int = 16
    d_conv: int = 4
    dt_rank: int = 32
    dt_init: float = 0.01


@dataclass(frozen=True)
class SmolVLASpec:
    """SmolVLA-shaped flow action expert (the reference's
    src/core/models/smolvla/smolvla_action_expert.cc:70-208 tensor set).

    `cache_width` is the width of the caller's per-layer prefix K / V cache:
    cross-attention layers project it (k_proj / v_proj take `cache_width`
    inputs) and self-attention layers attend over it directly when it equals
    `kv_heads * head_width` (the reference's layout), else over the action
    tokens only.
    """

    expert_width: int = 720
    layers: int = 16
    heads: int = 12
    kv_heads: int = 4
    head_width: int = 60
    mlp_width: int = 2048
    action_dim: int = 32
    chunk: int = 50
    state_dim: int = 32
    vlm_width: int = 960
    cache_width: int = 960
    prefix: int = 241

    @property
    def attention_width(self) -> int:
        return self.heads * self.head_width

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_width


# SmolVLA-shaped expert workload: 16 layers, width 720, 12 heads of 60, SwiGLU 2048, 50
# action tokens of dim 32, a 241-token prefix of width 960 projected per
# cross-attention layer (3:1 grouped-query attention, 4 K / V heads).
SMOLVLA_C5 = SmolVLASpec()
# The shapes the reference's loader accepts (smolvla_action_expert.cc:120-128:
# attention 960 = 15 x 64, K / V 320 = 5 x 64, MLP 2048, cache width 320).
SMOLVLA_REF = SmolVLASpec(expert_width=720, layers=4, heads=15, kv_heads=5, head_width=64, mlp_width=2048,
                          action_dim=32, chunk=10, state_dim=32, vlm_width=960, cache_width=320, prefix=24)

# PushT-shaped U-Net (A 2, H 16, cond 132).
PUSHT = DiffusionSpec(action_dim=2, horizon=16, condition_dim=132)
# bimanual U-Net (A 14, H 64, cond 284).
BIMANUAL = DiffusionSpec(action_dim=14, horizon=64, condition_dim=284, action_steps=32)
FLOW_C2 = FlowSpec()
MAMBA_C3 = MambaSpec()


class _Init:
    """PyTorch-default initialisation drawn from one seeded numpy stream."""

    def __init__(self, seed: int):
        self.rng = np.random.default_rng(seed)

    def uniform(self, shape, fan_in: int) -> np.ndarray:
        bound = np.float32(1.0 / math.sqrt(fan_in))
        unit = self.rng.random(size=shape, dtype=np.float32)
        return (unit * np.float32(2.0) - np.float32(1.0)) * bound

    def normal(self, shape) -> np.ndarray:
        return self.rng.standard_normal(size=shape, dtype=np.float32)


def _canonical(value) -> str:
    return json.dumps(value, ensure_ascii=True, sort_keys=True, separators=(",", ":"))


def diffusion_tensors(spec: DiffusionSpec, seed: int = 0):
    """Random-init ConditionalUnet1D in `dp.*` layout -> (tensors, metadata).

    Tensor names and shapes follow convert/convert.py:499-574; the U-Net
    structure follows LeRobot's ConditionalUnet1d as restated in the
    reference's tools/verification/verify_diffusion.py:18-127.
    """
    init = _Init(seed)
    a, k, td = spec.action_dim, spec.kernel, spec.timestep_dim
    film_width = td + spec.condition_dim
    out: dict = {}

    def conv(name, oc, ic, size):
        out[f"{name}.w"] = init.uniform((oc, ic, size), ic * size)
        out[f"{name}.b"] = init.uniform((oc,), ic * size)

    def linear(name, of, inf):
        out[f"{name}.w"] = init.uniform((of, inf), inf)
        out[f"{name}.b"] = init.uniform((of,), inf)

    def norm(name, ch):
        out[f"{name}.w"] = np.ones(ch, np.float32)
        out[f"{name}.b"] = np.zeros(ch, np.float32)

    def residual(name, ic, oc):
        conv(f"{name}.c1", oc, ic, k)
        norm(f"{name}.n1", oc)
        linear(f"{name}.film", 2 * oc, film_width)
        conv(f"{name}.c2", oc, oc, k)
        norm(f"{name}.n2", oc)
        if ic != oc:
            conv(f"{name}.res", oc, ic, 1)

    dims = list(spec.down_dims)
    linear("dp.te1", td * 4, td)
    linear("dp.te2", td, td * 4)
    for stage, oc in enumerate(dims):
        ic = a if stage == 0 else dims[stage - 1]
        residual(f"dp.d{stage}.r0", ic, oc)
        residual(f"dp.d{stage}.r1", oc, oc)
        if stage + 1 < len(dims):
            conv(f"dp.d{stage}.ds", oc, oc, 3)
    for block in range(2):
        residual(f"dp.m{block}", dims[-1], dims[-1])
    for stage in range(len(dims) - 1):
        high, low = dims[-1 - stage], dims[-2 - stage]
        residual(f"dp.u{stage}.r0", 2 * high, low)
        residual(f"dp.u{stage}.r1", low, low)
        # ConvTranspose1d storage is [in, out, k]; PyTorch's fan_in for it is
        # weight.size(1) * k = out * k.
        out[f"dp.u{stage}.us.w"] = init.uniform((low, low, 4), low * 4)
        out[f"dp.u{stage}.us.b"] = init.uniform((low,), low * 4)
    conv("dp.f.c", dims[0], dims[0], k)
    norm("dp.f.n", dims[0])
    conv("dp.f.o", a, dims[0], 1)
    amin = np.asarray(spec.action_min if spec.action_min else [-1.0] * a, np.float32)
    amax = np.asarray(spec.action_max if spec.action_max else [1.0] * a, np.float32)
    out["dp.action_min"] = amin
    out["dp.action_max"] = amax
    out["dp.dims"] = np.asarray(dims, np.float32)
    out["dp.meta"] = np.asarray(
        [1, a, spec.horizon, spec.action_steps, spec.observation_steps,
         spec.condition_dim, len(dims), k, spec.groups, td, spec.train_timesteps,
         0, 0, int(spec.clip_sample), spec.clip_sample_range, 0],
        np.float32,
    )
    schema = {"condition_dim": spec.condition_dim, "input_features": {},
              "observation_steps": spec.observation_steps}
    profile = {
        "profile_version": 1,
        "model_compatibility_version": 1,
        "observation_schema_hash": "sha256:" + hashlib.sha256(_canonical(schema).encode()).hexdigest(),
        "action_dim": a,
        "action_horizon": spec.horizon,
        "action_units": "physical",
        "normalization_type": "minmax",
        "normalization_parameters": {"min": amin.tolist(), "max": amax.tolist()},
        "solver_default": "euler",
        "solver_min_steps": 1,
        "solver_max_steps": min(spec.train_timesteps, 4096),
    }
    return out, {"flowedge.deployment_profile": _canonical(profile)}


def flow_tensors(spec: FlowSpec, seed: int = 0) -> dict:
    """Random-init flow velocity MLP (`flow.*`, no biases; flow.cc:64-98)."""
    init = _Init(seed)
    h = spec.hidden
    out = {
        "flow.in_proj.weight": init.uniform((h, spec.action_dim), spec.action_dim),
        "flow.time_proj.weight": init.uniform((h, spec.time_dim), spec.time_dim),
        "flow.cond_proj.weight": init.uniform((h, spec.cond_dim), spec.cond_dim),
    }
    for layer in range(spec.layers):
        out[f"flow.layers.{layer}.weight"] = init.uniform((h, h), h)
    out["flow.out_proj.weight"] = init.uniform((spec.action_dim, h), h)
    return out


def mamba_tensors(spec: MambaSpec, seed: int = 0) -> dict:
    """Random-init Mamba encoder in HF names (`backbone.*`; mamba.cc:103-222).

    A_log = log(1..d_state) per channel, D = 1, RMSNorm weights 1, dt bias =
    softplus^-1(dt_init), embedding table ~ N(0, 1).
    """
    init = _Init(seed)
    dm, di, ds, dc, dr = spec.d_model, spec.d_inner, spec.d_state, spec.d_conv, spec.dt_rank
    out = {"backbone.embeddings.weight": init.normal((spec.vocab, dm))}
    a_log = np.log(np.tile(np.arange(1, ds + 1, dtype=np.float32), (di, 1))).astype(np.float32)
    dt_bias = np.float32(math.log(math.expm1(spec.dt_init)))
    for layer in range(spec.n_layers):
        p = f"backbone.layers.{layer}."
        out[p + "norm.weight"] = np.ones(dm, np.float32)
        out[p + "mixer.in_proj.weight"] = init.uniform((2 * di, dm), dm)
        out[p + "mixer.conv1d.weight"] = init.uniform((di, 1, dc), dc)
        out[p + "mixer.conv1d.bias"] = init.uniform((di,), dc)
        out[p + "mixer.x_proj.weight"] = init.uniform((dr + 2 * ds, di), di)
        out[p + "mixer.dt_proj.weight"] = init.uniform((di, dr), dr)
        out[p + "mixer.dt_proj.bias"] = np.full(di, dt_bias, np.float32)
        out[p + "mixer.A_log"] = a_log.copy()
        out[p + "mixer.D"] = np.ones(di, np.float32)
        out[p + "mixer.out_proj.weight"] = init.uniform((dm, di), di)
    out["backbone.norm_f.weight"] = np.ones(dm, np.float32)
    return out


def smolvla_tensors(spec: SmolVLASpec, seed: int = 0) -> dict:
    """Random-init SmolVLA action expert (names and shapes of
    smolvla_action_expert.cc:70-180; Linear weights and biases PyTorch-default
    uniform, RMSNorm weights 1).  The matrices are rounded to bf16 values (the
    expert's source dtype); biases stay f32, as the reference loader requires
    (smolvla_action_expert.cc:98-105).  `flowedge.smolvla.head_width` records
    the head width, which the reference fixes at 64 and this build reads."""
    init = _Init(seed)
    w, a = spec.expert_width, spec.action_dim

    def lin(rows, cols):
        return bf16_bits_to_f32(to_bf16_bits(init.uniform((rows, cols), cols)))

    out = {
        "model.action_in_proj.weight": lin(w, a),
        "model.action_in_proj.bias": init.uniform((w,), a),
        "model.action_out_proj.weight": lin(a, w),
        "model.action_out_proj.bias": init.uniform((a,), w),
        "model.action_time_mlp_in.weight": lin(w, 2 * w),
        "model.action_time_mlp_in.bias": init.uniform((w,), 2 * w),
        "model.action_time_mlp_out.weight": lin(w, w),
        "model.action_time_mlp_out.bias": init.uniform((w,), w),
        "model.state_proj.weight": lin(spec.vlm_width, spec.state_dim),
        "model.state_proj.bias": init.uniform((spec.vlm_width,), spec.state_dim),
        "model.vlm_with_expert.lm_expert.norm.weight": np.ones(w, np.float32),
        "flowedge.smolvla.head_width": np.array([spec.head_width], np.float32),
    }
    for layer in range(spec.layers):
        p = f"model.vlm_with_expert.lm_expert.layers.{layer}."
        kv_in = spec.cache_width if layer % 2 == 1 else w
        out[p + "input_layernorm.weight"] = np.ones(w, np.float32)
        out[p + "post_attention_layernorm.weight"] = np.ones(w, np.float32)
        out[p + "self_attn.q_proj.weight"] = lin(spec.attention_width, w)
        out[p + "self_attn.k_proj.weight"] = lin(spec.kv_width, kv_in)
        out[p + "self_attn.v_proj.weight"] = lin(spec.kv_width, kv_in)
        out[p + "self_attn.o_proj.weight"] = lin(w, spec.attention_width)
        out[p + "mlp.gate_proj.weight"] = lin(spec.mlp_width, w)
        out[p + "mlp.up_proj.weight"] = lin(spec.mlp_width, w)
        out[p + "mlp.down_proj.weight"] = lin(w, spec.mlp_width)
    return out


def smolvla_prefix(spec: SmolVLASpec, seed: int = 0, batch: int | None = None, masked: int = 0):
    """Synthetic VLM prefix cache: keys and values [layers][prefix][cache_width]
    (with a leading batch axis when `batch` is given), bf16-valued ~N(0, 1),
    and a validity mask with the last `masked` slots padded."""
    rng = np.random.default_rng(seed)
    lead = () if batch is None else (batch,)
    shape = lead + (spec.layers, spec.prefix, spec.cache_width)
    keys = bf16_bits_to_f32(to_bf16_bits(rng.standard_normal(shape, dtype=np.float32)))
    values = bf16_bits_to_f32(to_bf16_bits(rng.standard_normal(shape, dtype=np.float32)))
    mask = np.ones(lead + (spec.prefix,), np.uint8)
    if masked:
        mask[..., spec.prefix - masked:] = 0
    return keys, values, mask


def cast_tensors(tensors: dict, matrices: str = "f32", convs: str = "f32") -> dict:
    """Apply the converter's dtype rule (2-D weights, convert.py:602-610) and,
    optionally, this build's BF16 conv mode (3-D `dp.*` conv weights)."""
    out = {}
    for name, value in tensors.items():
        bf16 = False
        if value.ndim == 2 and matrices == "bf16":
            bf16 = name != "backbone.embeddings.weight" and not name.endswith("mixer.A_log")
        if value.ndim == 3 and convs == "bf16" and name.startswith("dp."):
            bf16 = True
        out[name] = ("BF16", to_bf16_bits(value)) if bf16 else value
    return out


def recast_convs_bf16(src, dst, *, max_batch: int | None = None) -> dict:
    """Re-emit a converted checkpoint (e.g. one written by the reference's
    convert/convert.py) with its U-Net conv weights in BF16.

    The reference converter casts only 2-D tensors (convert.py:602-610), so its
    files hold every 3-D `dp.*` conv weight (conv [out][in][k], conv-transpose
    [in][out][4]) as F32.  This rewrites those tensors as BF16 (round to nearest
    even), copies every other tensor's bytes and dtype unchanged, keeps the
    file's metadata, and with `max_batch` adds the metadata key
    "flowedge.max_batch", which this library's loader takes as the engine's
    default batch reservation.  Returns {tensor name: "BF16"} for the recast
    tensors.
    """
    data = Path(src).read_bytes()
    (length,) = struct.unpack("<Q", data[:8])
    header = json.loads(data[8:8 + length])
    base = 8 + length
    metadata = dict(header.pop("__metadata__", {}))
    if max_batch is not None:
        if not 1 <= int(max_batch) <= 1 << 24:
            raise ValueError("max_batch must be from 1 through 16777216")
        metadata["flowedge.max_batch"] = str(int(max_batch))
    tensors, recast = {}, {}
    for name, entry in sorted(header.items(), key=lambda kv: kv[1]["data_offsets"][0]):
        begin, end = entry["data_offsets"]
        raw = data[base + begin:base + end]
        shape = tuple(entry["shape"])
        if entry["dtype"] == "F32" and len(shape) == 3 and name.startswith("dp."):
            tensors[name] = ("BF16", to_bf16_bits(np.frombuffer(raw, np.float32).reshape(shape)))
            recast[name] = "BF16"
        elif entry["dtype"] in ("F32", "BF16"):
            dt = np.float32 if entry["dtype"] == "F32" else np.uint16
            tensors[name] = (entry["dtype"], np.frombuffer(raw, dt).reshape(shape))
        else:
            raise ValueError(f"unsupported dtype {entry['dtype']} for {name}")
    write_safetensors(dst, tensors, metadata)
    return recast


def write_checkpoint(path, *parts, matrices: str = "f32", convs: str = "f32",
                     metadata: dict | None = None) -> Path:
    merged: dict = {}
    for part in parts:
        merged.update(part)
    write_safetensors(path, cast_tensors(merged, matrices, convs), metadata)
    return Path(path)


def _main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(prog="python -m flowedge_b200.checkpoint")
    sub = ap.add_subparsers(dest="cmd", required=True)
    rc = sub.add_parser("recast-convs", help="re-emit a converted checkpoint with BF16 U-Net conv weights")
    rc.add_argument("src")
    rc.add_argument("dst")
    rc.add_argument("--max-batch", type=int, default=None,
                    help="default batch reservation recorded in the file's metadata")
    args = ap.parse_args(argv)
    recast = recast_convs_bf16(args.src, args.dst, max_batch=args.max_batch)
    print(f"{args.dst}: {len(recast)} conv tensors as BF16")
    return 0


if __name__ == "__main__":
    raise SystemExit(_main())
