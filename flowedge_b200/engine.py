"""Python binding over libflowedge_b200.so (ctypes).

Mirrors the reference's pybind11 module (python/flowedge_ext.cc:790-856):
`Engine(path, threads=None)` with `sample_diffusion`, `diffusion_denoise`,
`sample`, `sample_condition`, `run`, `step`, `reset`, `decode_state`,
`restore_decode_state`, `flow_begin`, `flow_advance`, `cancel_before` and the
metadata properties, plus the batched methods this build adds.  Errors raise
RuntimeError carrying `fe_engine_last_error()` and the status code, as the
reference binding does.

There is no fallback: the library must be built (`python -m flowedge_b200.build`)
and a B200 must be present to create an engine.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libflowedge_b200.so"

_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)
_size_p = C.POINTER(C.c_size_t)
_u8p = C.POINTER(C.c_uint8)

SOLVERS = {"euler": 0, "heun": 1, "rk4": 2}
SCHEDULERS = {"ddim": 0, "ddpm": 1}
PRECISIONS = {"auto": 0, "fp32": 1, "bf16": 2}


class ModelMetadata(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("protocol_version", C.c_uint32),
                ("architecture", C.c_uint32), ("precision", C.c_uint32), ("model_digest", C.c_uint8 * 16),
                ("d_model", C.c_uint64), ("n_layers", C.c_uint64), ("d_inner", C.c_uint64),
                ("d_state", C.c_uint64), ("d_conv", C.c_uint64), ("action_dim", C.c_uint64),
                ("condition_dim", C.c_uint64), ("decode_snapshot_bytes", C.c_uint64)]


class DiffusionMetadata(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("protocol_version", C.c_uint32), ("clip_sample", C.c_uint32),
                ("reserved", C.c_uint32), ("action_dim", C.c_uint64), ("condition_dim", C.c_uint64),
                ("horizon", C.c_uint64), ("action_steps", C.c_uint64), ("observation_steps", C.c_uint64),
                ("train_timesteps", C.c_uint64), ("clip_sample_range", C.c_float),
                ("reserved_float", C.c_float)]


class ConditionMetadata(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("protocol_version", C.c_uint32), ("solver", C.c_uint32),
                ("reserved", C.c_uint32), ("model_digest", C.c_uint8 * 16), ("timestamp_ns", C.c_uint64),
                ("deadline_ns", C.c_uint64), ("generation", C.c_uint64), ("condition_dim", C.c_uint64),
                ("action_dim", C.c_uint64), ("solver_steps", C.c_uint64), ("remaining_nfe", C.c_uint64)]


class ActionMetadata(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("protocol_version", C.c_uint32), ("solver", C.c_uint32),
                ("status", C.c_uint32), ("model_digest", C.c_uint8 * 16), ("timestamp_ns", C.c_uint64),
                ("deadline_ns", C.c_uint64), ("generation", C.c_uint64), ("condition_dim", C.c_uint64),
                ("action_dim", C.c_uint64), ("remaining_nfe", C.c_uint64)]


class EngineOptions(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("worker_threads", C.c_uint32), ("device", C.c_int32),
                ("precision", C.c_uint32), ("max_batch", C.c_uint64), ("max_sequence", C.c_uint64)]


# name -> (restype, argtypes) for every entry point of include/flowedge_b200.h
SIGNATURES = {
    "fe_engine_last_error": (C.c_char_p, []),
    "fe_engine_load": (C.c_void_p, [C.c_char_p]),
    "fe_engine_load_with_threads": (C.c_void_p, [C.c_char_p, C.c_uint]),
    "fe_weights_load": (C.c_void_p, [C.c_char_p]),
    "fe_weights_size_bytes": (C.c_size_t, [C.c_void_p]),
    "fe_weights_free": (None, [C.c_void_p]),
    "fe_engine_create_from_weights": (C.c_void_p, [C.c_void_p, C.c_uint]),
    "fe_engine_create_from_weights_auto": (C.c_void_p, [C.c_void_p]),
    "fe_engine_dims": (None, [C.c_void_p, _size_p, _size_p]),
    "fe_engine_run": (C.c_int, [C.c_void_p, _i32p, C.c_size_t, _f32p]),
    "fe_engine_run_embeddings": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, _f32p]),
    "fe_engine_run_embeddings_masked": (C.c_int, [C.c_void_p, _f32p, C.c_void_p, C.c_size_t, _f32p]),
    "fe_engine_smolvla_embed_suffix": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, C.c_float, _f32p]),
    "fe_engine_smolvla_run_expert": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, _f32p, _f32p, C.c_void_p,
                                               C.c_size_t, _f32p]),
    "fe_engine_smolvla_project_actions": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, _f32p]),
    "fe_engine_smolvla_denoise": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, C.c_float, _f32p, _f32p, C.c_void_p,
                                            C.c_size_t, _f32p]),
    "fe_engine_smolvla_sample": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, C.c_size_t, _f32p, _f32p, C.c_void_p,
                                           C.c_size_t, _f32p]),
    "fe_engine_step": (C.c_int, [C.c_void_p, C.c_int32, _f32p]),
    "fe_engine_reset": (None, [C.c_void_p]),
    "fe_engine_thread_count": (C.c_uint, [C.c_void_p]),
    "fe_engine_cuda_resident": (C.c_int, [C.c_void_p]),
    "fe_engine_model_metadata": (C.c_int, [C.c_void_p, C.POINTER(ModelMetadata)]),
    "fe_engine_deployment_profile": (C.c_int, [C.c_void_p, C.c_void_p]),
    "fe_engine_action_dim": (C.c_size_t, [C.c_void_p]),
    "fe_engine_action_horizon": (C.c_size_t, [C.c_void_p]),
    "fe_engine_diffusion_metadata": (C.c_int, [C.c_void_p, C.POINTER(DiffusionMetadata)]),
    "fe_engine_condition_dim": (C.c_size_t, [C.c_void_p]),
    "fe_engine_sample_diffusion": (C.c_int, [C.c_void_p, _f32p, _f32p, C.c_size_t, C.c_int, C.c_uint64, _f32p]),
    "fe_engine_diffusion_denoise": (C.c_int, [C.c_void_p, _f32p, _f32p, C.c_float, _f32p]),
    "fe_engine_sample": (C.c_int, [C.c_void_p, _i32p, C.c_size_t, _f32p, C.c_size_t, C.c_int, _f32p]),
    "fe_engine_sample_condition": (C.c_int, [C.c_void_p, _f32p, _f32p, C.c_size_t, C.c_int, _f32p]),
    "fe_engine_flow_begin": (C.c_int, [C.c_void_p, _f32p, _f32p, C.c_size_t, C.c_int]),
    "fe_engine_make_condition_metadata": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_size_t,
                                                    C.c_int, C.POINTER(ConditionMetadata)]),
    "fe_engine_flow_begin_request": (C.c_int, [C.c_void_p, _f32p, _f32p, C.POINTER(ConditionMetadata)]),
    "fe_engine_cancel_before": (None, [C.c_void_p, C.c_uint64]),
    "fe_engine_flow_advance": (C.c_int, [C.c_void_p, C.c_size_t, _f32p, _size_p]),
    "fe_engine_flow_action_metadata": (C.c_int, [C.c_void_p, C.POINTER(ActionMetadata)]),
    "fe_engine_decode_state_bytes": (C.c_size_t, [C.c_void_p]),
    "fe_engine_export_decode_state": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "fe_engine_import_decode_state": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "fe_engine_free": (None, [C.c_void_p]),
    "fe_engine_smolvla_embed_suffix": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, C.c_float, _f32p]),
    "fe_engine_smolvla_run_expert": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, _f32p, _f32p, _u8p, C.c_size_t,
                                               _f32p]),
    "fe_engine_smolvla_project_actions": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, _f32p]),
    "fe_engine_smolvla_denoise": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, C.c_float, _f32p, _f32p, _u8p,
                                            C.c_size_t, _f32p]),
    "fe_engine_smolvla_sample": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, C.c_size_t, _f32p, _f32p, _u8p,
                                           C.c_size_t, _f32p]),
    # extensions
    "fe_engine_load_with_options": (C.c_void_p, [C.c_char_p, C.POINTER(EngineOptions)]),
    "fe_engine_create_from_weights_with_options": (C.c_void_p, [C.c_void_p, C.POINTER(EngineOptions)]),
    "fe_engine_reserve_batch": (C.c_int, [C.c_void_p, C.c_size_t]),
    "fe_engine_sample_diffusion_batch": (C.c_int, [C.c_void_p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_int,
                                                   C.c_uint64, _f32p]),
    "fe_engine_diffusion_denoise_batch": (C.c_int, [C.c_void_p, _f32p, _f32p, C.c_size_t, C.c_float, _f32p]),
    "fe_engine_sample_diffusion_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t,
                                                    C.c_int, C.c_uint64, C.c_void_p, C.c_void_p]),
    "fe_engine_sample_condition_batch": (C.c_int, [C.c_void_p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_int,
                                                   _f32p]),
    "fe_engine_sample_condition_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t,
                                                    C.c_int, C.c_void_p, C.c_void_p]),
    "fe_engine_sample_condition_static": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t,
                                                    C.c_int, C.c_void_p, C.c_void_p]),
    "fe_engine_run_batch": (C.c_int, [C.c_void_p, _i32p, C.c_size_t, C.c_size_t, _f32p]),
    "fe_engine_run_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p]),
    "fe_engine_sample_batch": (C.c_int, [C.c_void_p, _i32p, C.c_size_t, C.c_size_t, _f32p, C.c_size_t, C.c_int,
                                         _f32p]),
    "fe_engine_smolvla_sample_batch": (C.c_int, [C.c_void_p, _f32p, C.c_size_t, C.c_size_t, C.c_size_t, _f32p,
                                                 _f32p, _u8p, C.c_size_t, C.c_int, _f32p]),
    "fe_engine_smolvla_sample_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                                                  C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                                  C.c_void_p, C.c_void_p]),
    "fe_engine_smolvla_reserve": (C.c_int, [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int]),
    "fe_engine_synchronize": (C.c_int, [C.c_void_p]),
    "fe_engine_profile_diffusion": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_double)]),
    "fe_device_malloc_count": (C.c_uint64, []),
    "fe_host_malloc_count": (C.c_uint64, []),
    "fe_engine_kernel_launches": (C.c_uint64, [C.c_void_p]),
}

_lib = None


def load_library(path: str | Path | None = None):
    """Load the C-ABI library (raises if it was not built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    target = Path(path) if path else LIB_PATH
    if not target.exists():
        raise RuntimeError(f"{target} is not built; run `python -m flowedge_b200.build`")
    handle = C.CDLL(str(target))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if path is None:
        _lib = handle
    return handle


def _p(a):
    return a.ctypes.data_as(_f32p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class FlowEdgeError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"FlowEdge status {status}: {message}")
        self.status = status


class Engine:
    """One engine on one GPU (the reference `flowedge.Engine`)."""

    def __init__(self, path, threads: int | None = None, *, device: int | None = None, precision: str = "auto",
                 max_batch: int = 0, max_sequence: int = 0):
        self.lib = load_library()
        opts = EngineOptions(C.sizeof(EngineOptions), 0 if threads is None else threads,
                             -1 if device is None else device, PRECISIONS[precision], max_batch, max_sequence)
        self.handle = self.lib.fe_engine_load_with_options(str(path).encode(), C.byref(opts))
        if not self.handle:
            raise RuntimeError(self.lib.fe_engine_last_error().decode())

    # ---- lifetime
    def close(self):
        if getattr(self, "handle", None):
            self.lib.fe_engine_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def _check(self, rc: int):
        if rc != 0:
            raise FlowEdgeError(rc, self.lib.fe_engine_last_error().decode())

    # ---- metadata
    @property
    def action_dim(self) -> int:
        return self.lib.fe_engine_action_dim(self.handle)

    @property
    def action_horizon(self) -> int:
        return self.lib.fe_engine_action_horizon(self.handle)

    @property
    def condition_dim(self) -> int:
        return self.lib.fe_engine_condition_dim(self.handle)

    @property
    def d_model(self) -> int:
        d, n = C.c_size_t(), C.c_size_t()
        self.lib.fe_engine_dims(self.handle, C.byref(d), C.byref(n))
        return d.value

    @property
    def thread_count(self) -> int:
        return self.lib.fe_engine_thread_count(self.handle)

    @property
    def cuda_resident(self) -> bool:
        return bool(self.lib.fe_engine_cuda_resident(self.handle))

    @property
    def model_metadata(self) -> dict:
        m = ModelMetadata()
        self._check(self.lib.fe_engine_model_metadata(self.handle, C.byref(m)))
        out = {name: getattr(m, name) for name, _ in ModelMetadata._fields_}
        out["model_digest"] = bytes(m.model_digest)
        return out

    @property
    def diffusion_metadata(self) -> dict:
        m = DiffusionMetadata()
        self._check(self.lib.fe_engine_diffusion_metadata(self.handle, C.byref(m)))
        return {"protocol_version": m.protocol_version, "action_dim": m.action_dim,
                "condition_dim": m.condition_dim, "horizon": m.horizon, "action_steps": m.action_steps,
                "observation_steps": m.observation_steps, "train_timesteps": m.train_timesteps,
                "clip_sample": bool(m.clip_sample), "clip_sample_range": m.clip_sample_range}

    @property
    def flow_metadata(self) -> dict:
        m = ActionMetadata()
        self._check(self.lib.fe_engine_flow_action_metadata(self.handle, C.byref(m)))
        out = {name: getattr(m, name) for name, _ in ActionMetadata._fields_}
        out["model_digest"] = bytes(m.model_digest)
        return out

    @property
    def kernel_launches(self) -> int:
        return self.lib.fe_engine_kernel_launches(self.handle)

    # ---- Diffusion Policy
    def sample_diffusion(self, condition, noise, steps: int = 10, scheduler: str = "ddim", seed: int = 0):
        cond, x = _f32(condition), _f32(noise)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_sample_diffusion(self.handle, _p(cond), _p(x), steps,
                                                        SCHEDULERS[scheduler], seed, _p(out)))
        return out

    def sample_diffusion_into(self, condition, noise, output, steps: int = 10, scheduler: str = "ddim",
                              seed: int = 0):
        cond, x = _f32(condition), _f32(noise)
        assert output.dtype == np.float32 and output.flags.c_contiguous and output.size == x.size
        self._check(self.lib.fe_engine_sample_diffusion(self.handle, _p(cond), _p(x), steps,
                                                        SCHEDULERS[scheduler], seed, _p(output)))

    def diffusion_denoise(self, condition, sample, timestep: float):
        cond, x = _f32(condition), _f32(sample)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_diffusion_denoise(self.handle, _p(cond), _p(x), float(timestep), _p(out)))
        return out

    def sample_diffusion_batch(self, condition, noise, steps: int = 10, scheduler: str = "ddim", seed: int = 0):
        cond, x = _f32(condition), _f32(noise)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_sample_diffusion_batch(self.handle, _p(cond), _p(x), x.shape[0], steps,
                                                              SCHEDULERS[scheduler], seed, _p(out)))
        return out

    def diffusion_denoise_batch(self, condition, sample, timestep: float):
        cond, x = _f32(condition), _f32(sample)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_diffusion_denoise_batch(self.handle, _p(cond), _p(x), x.shape[0],
                                                               float(timestep), _p(out)))
        return out

    def sample_diffusion_device(self, condition_ptr: int, noise_ptr: int, batch: int, action_ptr: int,
                                steps: int = 10, scheduler: str = "ddim", seed: int = 0, stream: int = 0):
        self._check(self.lib.fe_engine_sample_diffusion_device(
            self.handle, C.c_void_p(condition_ptr), C.c_void_p(noise_ptr), batch, steps, SCHEDULERS[scheduler],
            seed, C.c_void_p(action_ptr), C.c_void_p(stream or None)))

    def reserve_batch(self, max_batch: int):
        self._check(self.lib.fe_engine_reserve_batch(self.handle, max_batch))

    def profile_diffusion(self, batch: int) -> dict:
        m = (C.c_double * 4)()
        self._check(self.lib.fe_engine_profile_diffusion(self.handle, batch, m))
        return {"conv_ms": m[0], "conv_launches": int(m[1]), "conv_flops": m[2], "forward_ms": m[3]}

    def synchronize(self):
        self._check(self.lib.fe_engine_synchronize(self.handle))

    # ---- flow head
    def sample_condition(self, condition, noise, output=None, steps: int = 10, method: str = "euler"):
        cond, x = _f32(condition), _f32(noise)
        out = np.empty_like(x) if output is None else output
        self._check(self.lib.fe_engine_sample_condition(self.handle, _p(cond), _p(x), steps, SOLVERS[method],
                                                        _p(out)))
        return out

    def sample_condition_batch(self, condition, noise, steps: int = 10, method: str = "euler"):
        cond, x = _f32(condition), _f32(noise)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_sample_condition_batch(self.handle, _p(cond), _p(x), x.shape[0], steps,
                                                              SOLVERS[method], _p(out)))
        return out

    def sample_condition_device(self, condition_ptr: int, noise_ptr: int, batch: int, action_ptr: int,
                                steps: int = 10, method: str = "euler", stream: int = 0):
        self._check(self.lib.fe_engine_sample_condition_device(
            self.handle, C.c_void_p(condition_ptr), C.c_void_p(noise_ptr), batch, steps, SOLVERS[method],
            C.c_void_p(action_ptr), C.c_void_p(stream or None)))

    def flow_begin(self, condition, noise, steps: int = 10, method: str = "euler", generation=None,
                   timestamp_ns: int = 0, deadline_ns: int = 0):
        cond, x = _f32(condition), _f32(noise)
        if generation is None:
            self._check(self.lib.fe_engine_flow_begin(self.handle, _p(cond), _p(x), steps, SOLVERS[method]))
            return
        meta = ConditionMetadata()
        self._check(self.lib.fe_engine_make_condition_metadata(self.handle, timestamp_ns, deadline_ns, generation,
                                                               steps, SOLVERS[method], C.byref(meta)))
        self._check(self.lib.fe_engine_flow_begin_request(self.handle, _p(cond), _p(x), C.byref(meta)))

    def flow_advance(self, output, step_budget: int = 1) -> int:
        remaining = C.c_size_t()
        rc = self.lib.fe_engine_flow_advance(self.handle, step_budget, _p(output), C.byref(remaining))
        self._check(rc)
        return remaining.value

    def cancel_before(self, generation: int):
        self.lib.fe_engine_cancel_before(self.handle, generation)

    # ---- Mamba backbone
    def run(self, tokens):
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.empty((toks.size, self.d_model), np.float32)
        self._check(self.lib.fe_engine_run(self.handle, toks.ctypes.data_as(_i32p), toks.size, _p(out)))
        return out

    def run_device(self, tokens_ptr: int, batch: int, seq_len: int, last_hidden_ptr: int, stream: int = 0):
        """Prefill on device buffers (last hidden state of each sequence); asynchronous."""
        self._check(self.lib.fe_engine_run_device(self.handle, tokens_ptr, batch, seq_len, last_hidden_ptr,
                                                  stream or None))

    def run_batch(self, tokens):
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.empty((toks.shape[0], toks.shape[1], self.d_model), np.float32)
        self._check(self.lib.fe_engine_run_batch(self.handle, toks.ctypes.data_as(_i32p), toks.shape[0],
                                                 toks.shape[1], _p(out)))
        return out

    def sample(self, prefix, noise, steps: int = 10, method: str = "euler"):
        toks = np.ascontiguousarray(prefix, np.int32)
        x = _f32(noise)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_sample(self.handle, toks.ctypes.data_as(_i32p), toks.size, _p(x), steps,
                                              SOLVERS[method], _p(out)))
        return out

    def sample_batch(self, tokens, noise, steps: int = 10, method: str = "euler"):
        toks = np.ascontiguousarray(tokens, np.int32)
        x = _f32(noise)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_sample_batch(self.handle, toks.ctypes.data_as(_i32p), toks.shape[0],
                                                    toks.shape[1], _p(x), steps, SOLVERS[method], _p(out)))
        return out

    def step(self, token: int):
        out = np.empty(self.d_model, np.float32)
        self._check(self.lib.fe_engine_step(self.handle, int(token), _p(out)))
        return out

    def reset(self):
        self.lib.fe_engine_reset(self.handle)

    # ---- SmolVLA action expert (engine.h:136-196); prefix caches [layers][prefix][cache_width]
    @staticmethod
    def _u8(a):
        return a.ctypes.data_as(_u8p)

    def smolvla_embed_suffix(self, noisy, timestep: float, width: int):
        x = _f32(noisy)
        out = np.empty((x.shape[0], width), np.float32)
        self._check(self.lib.fe_engine_smolvla_embed_suffix(self.handle, _p(x), x.shape[0], float(timestep),
                                                            _p(out)))
        return out

    def smolvla_run_expert(self, suffix, keys, values, mask):
        x, k, v = _f32(suffix), _f32(keys), _f32(values)
        m = np.ascontiguousarray(mask, np.uint8)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_smolvla_run_expert(self.handle, _p(x), x.shape[0], _p(k), _p(v), self._u8(m),
                                                          m.size, _p(out)))
        return out

    def smolvla_project_actions(self, hidden):
        x = _f32(hidden)
        out = np.empty((x.shape[0], self.action_dim), np.float32)
        self._check(self.lib.fe_engine_smolvla_project_actions(self.handle, _p(x), x.shape[0], _p(out)))
        return out

    def smolvla_denoise(self, noisy, timestep: float, keys, values, mask):
        x, k, v = _f32(noisy), _f32(keys), _f32(values)
        m = np.ascontiguousarray(mask, np.uint8)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_smolvla_denoise(self.handle, _p(x), x.shape[0], float(timestep), _p(k), _p(v),
                                                       self._u8(m), m.size, _p(out)))
        return out

    def smolvla_sample(self, noise, steps: int, keys, values, mask):
        x, k, v = _f32(noise), _f32(keys), _f32(values)
        m = np.ascontiguousarray(mask, np.uint8)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_smolvla_sample(self.handle, _p(x), x.shape[0], steps, _p(k), _p(v),
                                                      self._u8(m), m.size, _p(out)))
        return out

    def smolvla_sample_batch(self, noise, steps: int, keys, values, mask, shared_prefix: bool = False):
        """noise [batch][chunk][A]; keys / values [batch][layers][prefix][cache_width] and mask
        [batch][prefix], or a single prefix ([layers][prefix][cache_width], [prefix]) when shared."""
        x, k, v = _f32(noise), _f32(keys), _f32(values)
        m = np.ascontiguousarray(mask, np.uint8)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_smolvla_sample_batch(self.handle, _p(x), x.shape[0], x.shape[1], steps, _p(k),
                                                            _p(v), self._u8(m), m.shape[-1], int(shared_prefix),
                                                            _p(out)))
        return out

    def smolvla_sample_device(self, noise_ptr: int, batch: int, chunk: int, steps: int, keys_ptr: int,
                              values_ptr: int, mask_ptr: int, prefix: int, shared_prefix: bool, out_ptr: int,
                              stream: int = 0):
        self._check(self.lib.fe_engine_smolvla_sample_device(self.handle, noise_ptr, batch, chunk, steps, keys_ptr,
                                                             values_ptr, mask_ptr, prefix, int(shared_prefix),
                                                             out_ptr, stream or None))

    def smolvla_reserve(self, batch: int, chunk: int, prefix: int, shared_prefix: bool = False):
        self._check(self.lib.fe_engine_smolvla_reserve(self.handle, batch, chunk, prefix, int(shared_prefix)))

    def decode_state(self) -> bytes:
        size = self.lib.fe_engine_decode_state_bytes(self.handle)
        buf = C.create_string_buffer(size)
        self._check(self.lib.fe_engine_export_decode_state(self.handle, buf, size))
        return buf.raw

    def restore_decode_state(self, snapshot: bytes):
        buf = C.create_string_buffer(bytes(snapshot), len(snapshot))
        self._check(self.lib.fe_engine_import_decode_state(self.handle, buf, len(snapshot)))


def device_malloc_count() -> int:
    return load_library().fe_device_malloc_count()


def host_malloc_count() -> int:
    return load_library().fe_host_malloc_count()
