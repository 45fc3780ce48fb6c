"""Pins the SmolVLA expert restatement (oracle/restate.py SmolVLAExpert) to the
reference's own outputs at the shapes its loader accepts.

tests/golden/make_golden.py ran the reference core (oracle/_ref) on checkpoints
and prefix caches that flowedge_b200.checkpoint regenerates here from the
stored (spec, seed).  The fp32 paths (suffix embedding, action projection)
agree to ~1e-6.  The expert layers round every intermediate to bf16, so a
change of summation order flips roundings that the next layers carry on: the
restatement with float64 instead of float32 matmuls moves the 16-layer hidden
state by ~1.4% relative, the same as its distance to the reference (~1.5%).
The layer outputs are therefore compared by relative L2 error, and the
10-step Euler sample by the bf16 parity bar (2e-2 max-abs).
"""

import dataclasses
import json

import numpy as np
import pytest

from flowedge_b200 import checkpoint as ck
from oracle import restate
from tests.conftest import GOLDEN


def smolvla_fixture(name):
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    p = json.loads(str(g["params"]))
    spec = dataclasses.replace(ck.SMOLVLA_REF, layers=p["layers"], chunk=p["chunk"], prefix=p["prefix"])
    tensors = ck.smolvla_tensors(spec, p["seed"])
    keys, values, mask = ck.smolvla_prefix(spec, p["seed"] + 1, masked=p["masked"])
    return spec, p, tensors, keys, values, mask, g


def rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("name", ["smolvla_ref", "smolvla_ref16"])
def test_smolvla_restatement_matches_reference(name):
    spec, p, tensors, keys, values, mask, g = smolvla_fixture(name)
    e = restate.SmolVLAExpert(tensors)
    assert (e.heads, e.kv_heads, e.head_width, e.cache_width) == (15, 5, 64, 320)
    np.testing.assert_allclose(e.embed_suffix(g["noise"], g["timestep"]), g["embed"], atol=1e-4)
    np.testing.assert_allclose(e.project_actions(g["hidden"]), g["project"], atol=1e-4)
    assert rel(e.run(g["embed"], keys, values, mask), g["hidden"]) < 3e-2
    assert rel(e.denoise(g["noise"], g["timestep"], keys, values, mask), g["denoise"]) < 3e-2
    sample = e.sample(g["noise"], p["steps"], keys, values, mask)
    assert float(np.abs(sample - g["sample"]).max()) <= 2e-2


def test_round_bf16_matches_bit_rule():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.0e-5, 65504.0, 1e-40], np.float32)
    bits = x.view(np.uint32)
    expect = ((bits + (((bits >> 16) & 1) + 0x7FFF)) & 0xFFFF0000).view(np.float32)
    np.testing.assert_array_equal(restate.round_bf16(x), expect)
    assert restate.round_bf16(np.array([1.00390625], np.float32))[0] == 1.0  # tie to even


def test_rope_preserves_pair_norms():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 3, 60)).astype(np.float32)
    y = restate.apply_rope(x, 60, 7)
    n0 = x[..., :30] ** 2 + x[..., 30:] ** 2
    n1 = y[..., :30] ** 2 + y[..., 30:] ** 2
    np.testing.assert_allclose(n1, n0, rtol=1e-5)
    np.testing.assert_allclose(restate.apply_rope(x, 60, 0)[0], x[0], atol=0)  # position 0 is the identity
