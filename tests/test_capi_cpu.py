"""Host-side checks that need no GPU: the library exports every symbol the
public headers declare, loading fails loudly without an sm_100 device, the
weight store and argument checks behave like the reference (src/core/api/engine.cc)."""

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from flowedge_b200 import engine as fe
from flowedge_b200 import checkpoint as ck

REPO = Path(__file__).resolve().parents[1]


def _declared(header):
    text = (REPO / "include" / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:fe|febtest)_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from flowedge_b200 import build

    build.build()
    return fe.load_library()


def test_every_declared_symbol_is_exported(lib):
    names = _declared("flowedge_b200.h") + _declared("flowedge_b200_testing.h")
    assert len(names) >= 56
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the binding's signature table covers the whole public header
    assert set(_declared("flowedge_b200.h")) <= set(fe.SIGNATURES)


def test_reference_abi_names_are_all_present():
    # the reference engine.h entry points (src/core/api/engine.h:63-395)
    reference = """fe_engine_last_error fe_engine_load fe_engine_load_with_threads fe_weights_load
    fe_weights_size_bytes fe_weights_free fe_engine_create_from_weights fe_engine_create_from_weights_auto
    fe_engine_dims fe_engine_run fe_engine_run_embeddings fe_engine_run_embeddings_masked
    fe_engine_smolvla_embed_suffix fe_engine_smolvla_run_expert fe_engine_smolvla_project_actions
    fe_engine_smolvla_denoise fe_engine_smolvla_sample fe_engine_step fe_engine_reset fe_engine_thread_count
    fe_engine_cuda_resident fe_engine_model_metadata fe_engine_deployment_profile fe_engine_action_dim
    fe_engine_action_horizon fe_engine_diffusion_metadata fe_engine_condition_dim fe_engine_sample_diffusion
    fe_engine_diffusion_denoise fe_engine_sample fe_engine_sample_condition fe_engine_flow_begin
    fe_engine_make_condition_metadata fe_engine_flow_begin_request fe_engine_cancel_before
    fe_engine_flow_advance fe_engine_flow_action_metadata fe_engine_decode_state_bytes
    fe_engine_export_decode_state fe_engine_import_decode_state fe_engine_free""".split()
    assert set(reference) <= set(_declared("flowedge_b200.h"))


def _has_gpu():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU failure path")
def test_load_without_gpu_fails_loudly(lib):
    h = lib.fe_engine_load_with_threads(str(REPO / "tests/golden/unet_tiny.safetensors").encode(), 0)
    assert not h
    assert b"no CUDA device" in lib.fe_engine_last_error()


def test_weights_store_and_errors(lib):
    w = lib.fe_weights_load(str(REPO / "tests/golden/unet_tiny.safetensors").encode())
    assert w
    tensors, _ = ck.read_safetensors(REPO / "tests/golden/unet_tiny.safetensors")
    assert lib.fe_weights_size_bytes(w) == sum(t.nbytes for t in tensors.values())
    lib.fe_weights_free(w)
    assert not lib.fe_weights_load(b"/nonexistent.safetensors")
    assert lib.fe_engine_last_error() == b"Failed to open safetensors file"
    assert not lib.fe_weights_load(None)
    assert lib.fe_engine_last_error() == b"Invalid null model path"
    assert lib.fe_engine_load_with_threads(b"x", 9) is None
    # null engine: status 1 with the reference's message (engine.cc:511-515)
    assert lib.fe_engine_sample_diffusion(None, None, None, 10, 0, 0, None) == 1
    assert lib.fe_engine_last_error() == b"Invalid arguments to fe_engine_sample_diffusion"
    assert lib.fe_engine_flow_advance(None, 1, None, None) == 1
    assert lib.fe_engine_action_dim(None) == 0 and lib.fe_engine_cuda_resident(None) == 0


def test_truncated_and_corrupt_files_are_rejected(lib, tmp_path):
    data = (REPO / "tests/golden/unet_tiny.safetensors").read_bytes()
    bad = tmp_path / "trunc.safetensors"
    bad.write_bytes(data[:-100])
    assert not lib.fe_weights_load(str(bad).encode())
    assert b"out of bounds" in lib.fe_engine_last_error()
    bad.write_bytes(b"\xff" * 8 + data[8:])
    assert not lib.fe_weights_load(str(bad).encode())
    assert lib.fe_engine_last_error() == b"Invalid header length"
    bad.write_bytes(b"\x00" * 4)
    assert not lib.fe_weights_load(str(bad).encode())


def test_checkpoint_writer_round_trip(tmp_path):
    spec = ck.DiffusionSpec(action_dim=2, horizon=8, condition_dim=6, down_dims=(16, 32), timestep_dim=8)
    tensors, meta = ck.diffusion_tensors(spec, seed=1)
    path = tmp_path / "a.safetensors"
    ck.write_checkpoint(path, tensors, metadata=meta, convs="bf16")
    back, md = ck.read_safetensors(path)
    assert md["flowedge.deployment_profile"] == meta["flowedge.deployment_profile"]
    for k, v in tensors.items():
        if v.ndim == 3:
            np.testing.assert_allclose(back[k], v, rtol=2 ** -8)
        else:
            np.testing.assert_array_equal(back[k], v)


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.5e-3, 65504.0], np.float32)
    bits = ck.to_bf16_bits(x)
    ref = __import__("torch").from_numpy(x).to(__import__("torch").bfloat16).view(__import__("torch").int16)
    np.testing.assert_array_equal(bits.view(np.int16), ref.numpy())


def test_gaussian_stream_random_access_matches_sequential():
    """The device generates DDPM noise by value index: draw k of a stream seeded
    with s mixes s + (k + 1) * golden; value j uses draws 2*(j//2)+1, 2*(j//2)+2
    (cosine for even j, sine for odd).  That equals the sequential host stream."""
    from oracle import restate

    golden = restate.GaussianGenerator.GOLDEN
    mask = restate.GaussianGenerator.MASK

    def mix(v):
        v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & mask
        v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & mask
        return v ^ (v >> 31)

    def at(seed, j):
        pair = j >> 1
        u = lambda k: np.float32(np.float32((mix((seed + (k + 1) * golden) & mask) >> 40) + 1) / np.float32(16777217.0))
        first = max(u(2 * pair + 1), np.finfo(np.float32).tiny)
        second = u(2 * pair + 2)
        r = np.sqrt(np.float32(-2.0) * np.log(np.float32(first)), dtype=np.float32)
        a = np.float32(np.float32(2 * np.pi) * second)
        return np.float32(r * (np.sin(a, dtype=np.float32) if j & 1 else np.cos(a, dtype=np.float32)))

    for seed in (0, 42, 2**63 + 5):
        seq = restate.GaussianGenerator(seed).fill(37)
        ra = np.array([at(seed, j) for j in range(37)], np.float32)
        np.testing.assert_array_equal(seq, ra)


def _fp16_check(lib, w, bf16_mode, name=b"dp.d0.r0.c1.w"):
    fn = lib.febtest_check_fp16_storable
    fn.restype = C.c_int
    fn.argtypes = [C.c_char_p, C.POINTER(C.c_float), C.c_size_t, C.c_int, C.c_char_p, C.c_size_t]
    w = np.ascontiguousarray(w, np.float32)
    msg = C.create_string_buffer(512)
    rc = fn(name, w.ctypes.data_as(C.POINTER(C.c_float)), w.size, int(bf16_mode), msg, len(msg))
    return rc, msg.value.decode()


@pytest.mark.parametrize("bf16_mode", [True, False])
def test_fp16_weight_storage_range_check(lib, bf16_mode):
    """Weights the device holds in fp16 (bf16 mode: fp16(bf16(w)); fp32 mode:
    fp16 hi + lo) are range-checked at load: a value beyond 65504, a non-finite
    value, or a tensor whose values all sit in fp16's subnormal range is
    rejected with a message naming the tensor; ordinary PyTorch-default inits
    (down to 1/sqrt(20480) for the widest conv) pass."""
    rng = np.random.default_rng(0)
    bound = 1.0 / np.sqrt(20480.0)
    ok = rng.uniform(-bound, bound, 4096).astype(np.float32)
    ok[:10] = 0.0  # exact zeros and tiny values inside an ordinary tensor are fine
    ok[10:20] = 1e-9
    assert _fp16_check(lib, ok, bf16_mode) == (0, "")
    # 65504 is fp16's largest value; bf16 rounds it up to 65536, beyond fp16
    assert _fp16_check(lib, np.array([65504.0, -3.0], np.float32), bf16_mode)[0] == (1 if bf16_mode else 0)
    big = ok.copy()
    big[123] = 70000.0
    rc, msg = _fp16_check(lib, big, bf16_mode)
    assert rc == 1 and "dp.d0.r0.c1.w" in msg and "65504" in msg and "123" in msg
    nan = ok.copy()
    nan[7] = np.nan
    rc, msg = _fp16_check(lib, nan, bf16_mode)
    assert rc == 1 and "non-finite" in msg
    tiny = (ok * 1e-6).astype(np.float32)  # every value below 2^-17: fp16 subnormals only
    rc, msg = _fp16_check(lib, tiny, bf16_mode)
    assert rc == 1 and "subnormal" in msg


def test_fp16_weight_storage_error_bounds_match_the_documented_split(lib):
    """fp32 mode's hi / lo pair is within max(2^-22 |w|, 2^-25) of w, so the
    check accepts a tensor of scale 2^-8 and rejects one of scale 2^-17."""
    rng = np.random.default_rng(1)
    w = rng.uniform(-1, 1, 8192).astype(np.float32) * np.float32(2.0 ** -8)
    assert _fp16_check(lib, w, False)[0] == 0
    assert _fp16_check(lib, w * np.float32(2.0 ** -9), False)[0] == 1


def test_recast_reference_converted_convs_to_bf16(lib, tmp_path):
    """A file written by the reference converter (the golden fixture, made by
    its convert/convert.py, which keeps 3-D convs F32) re-emitted with BF16
    conv weights: every 3-D dp.* tensor becomes the nearest-even bf16 of the
    original, every other tensor and the metadata are unchanged, the optional
    batch reservation lands in the metadata, and the loader accepts the file
    (and rejects a malformed reservation)."""
    src = REPO / "tests/golden/unet_small.safetensors"
    dst = tmp_path / "unet_small_bf16conv.safetensors"
    recast = ck.recast_convs_bf16(src, dst, max_batch=32)
    before, meta0 = ck.read_safetensors(src)
    after, meta1 = ck.read_safetensors(dst)
    convs = [k for k, v in before.items() if v.ndim == 3 and k.startswith("dp.")]
    assert sorted(recast) == sorted(convs) and len(convs) > 20
    for k, v in before.items():
        if k in recast:
            np.testing.assert_array_equal(after[k], ck.bf16_bits_to_f32(ck.to_bf16_bits(v)))
        else:
            np.testing.assert_array_equal(after[k], v)
    assert meta1 == dict(meta0, **{"flowedge.max_batch": "32"})
    w = lib.fe_weights_load(str(dst).encode())
    assert w
    w_src = lib.fe_weights_load(str(src).encode())
    assert lib.fe_weights_size_bytes(w) < lib.fe_weights_size_bytes(w_src)
    lib.fe_weights_free(w)
    lib.fe_weights_free(w_src)
    bad = tmp_path / "bad_meta.safetensors"
    t, m = ck.read_safetensors(src)
    ck.write_safetensors(bad, t, dict(m, **{"flowedge.max_batch": "0"}))
    assert not lib.fe_weights_load(str(bad).encode())
    assert b"flowedge.max_batch" in lib.fe_engine_last_error()
    with pytest.raises(ValueError):
        ck.recast_convs_bf16(src, tmp_path / "x.safetensors", max_batch=0)
