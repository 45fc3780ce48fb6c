"""ctypes binding to the reference FlowEdge core built by oracle/Makefile.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  The signatures follow the
reference C ABI, src/core/api/engine.h:63-395.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_ref" / "liboracle.so"
# the reference checkout, given by FLOWEDGE_REFERENCE (needed only to build)
REFERENCE_ROOT = Path(os.environ["FLOWEDGE_REFERENCE"]) if os.environ.get("FLOWEDGE_REFERENCE") else None

_f32p = C.POINTER(C.c_float)


def build(root: Path | None = None) -> Path:
    """Compile the reference core from the checkout at `root` (default:
    FLOWEDGE_REFERENCE) unless it is built already."""
    if not LIB_PATH.exists():
        root = root if root is not None else REFERENCE_ROOT
        if root is None or not (Path(root) / "src" / "core").is_dir():
            raise FileNotFoundError(f"{LIB_PATH} missing: set FLOWEDGE_REFERENCE to a reference checkout to build it")
        subprocess.run(["make", "-C", str(HERE), f"REF={root}", "-j8"], check=True, stdout=subprocess.DEVNULL)
    return LIB_PATH


def available() -> bool:
    return LIB_PATH.exists()


class _ModelMetadata(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("protocol_version", C.c_uint32),
                ("architecture", C.c_uint32), ("precision", C.c_uint32),
                ("digest", C.c_uint8 * 16), ("d_model", C.c_uint64), ("n_layers", C.c_uint64),
                ("d_inner", C.c_uint64), ("d_state", C.c_uint64), ("d_conv", C.c_uint64),
                ("action_dim", C.c_uint64), ("condition_dim", C.c_uint64),
                ("decode_snapshot_bytes", C.c_uint64)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        handle = C.CDLL(str(build()))
        handle.fe_engine_load_with_threads.restype = C.c_void_p
        handle.fe_engine_load_with_threads.argtypes = [C.c_char_p, C.c_uint]
        handle.fe_engine_free.argtypes = [C.c_void_p]
        handle.fe_weights_load.restype = C.c_void_p
        handle.fe_weights_load.argtypes = [C.c_char_p]
        handle.fe_weights_free.argtypes = [C.c_void_p]
        handle.fe_engine_create_from_weights.restype = C.c_void_p
        handle.fe_engine_create_from_weights.argtypes = [C.c_void_p, C.c_uint]
        handle.fe_engine_last_error.restype = C.c_char_p
        handle.fe_engine_sample_diffusion.argtypes = [C.c_void_p, _f32p, _f32p, C.c_size_t,
                                                      C.c_int, C.c_uint64, _f32p]
        handle.fe_engine_diffusion_denoise.argtypes = [C.c_void_p, _f32p, _f32p, C.c_float, _f32p]
        handle.fe_engine_sample_condition.argtypes = [C.c_void_p, _f32p, _f32p, C.c_size_t,
                                                      C.c_int, _f32p]
        handle.fe_engine_sample.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_size_t, _f32p,
                                            C.c_size_t, C.c_int, _f32p]
        handle.fe_engine_run.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_size_t, _f32p]
        handle.fe_engine_step.argtypes = [C.c_void_p, C.c_int32, _f32p]
        handle.fe_engine_reset.argtypes = [C.c_void_p]
        handle.fe_engine_model_metadata.argtypes = [C.c_void_p, C.POINTER(_ModelMetadata)]
        handle.fe_engine_decode_state_bytes.restype = C.c_size_t
        handle.fe_engine_decode_state_bytes.argtypes = [C.c_void_p]
        handle.fe_engine_export_decode_state.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
        handle.fe_engine_action_dim.restype = C.c_size_t
        handle.fe_engine_action_dim.argtypes = [C.c_void_p]
        handle.fe_engine_action_horizon.restype = C.c_size_t
        handle.fe_engine_action_horizon.argtypes = [C.c_void_p]
        handle.fe_engine_condition_dim.restype = C.c_size_t
        handle.fe_engine_condition_dim.argtypes = [C.c_void_p]
        handle.fe_engine_flow_begin.argtypes = [C.c_void_p, _f32p, _f32p, C.c_size_t, C.c_int]
        handle.fe_engine_flow_advance.argtypes = [C.c_void_p, C.c_size_t, _f32p,
                                                  C.POINTER(C.c_size_t)]
        _u8p = C.POINTER(C.c_uint8)
        handle.fe_engine_smolvla_embed_suffix.argtypes = [C.c_void_p, _f32p, C.c_size_t, C.c_float, _f32p]
        handle.fe_engine_smolvla_run_expert.argtypes = [C.c_void_p, _f32p, C.c_size_t, _f32p, _f32p, _u8p,
                                                        C.c_size_t, _f32p]
        handle.fe_engine_smolvla_project_actions.argtypes = [C.c_void_p, _f32p, C.c_size_t, _f32p]
        handle.fe_engine_smolvla_denoise.argtypes = [C.c_void_p, _f32p, C.c_size_t, C.c_float, _f32p, _f32p,
                                                     _u8p, C.c_size_t, _f32p]
        handle.fe_engine_smolvla_sample.argtypes = [C.c_void_p, _f32p, C.c_size_t, C.c_size_t, _f32p, _f32p,
                                                    _u8p, C.c_size_t, _f32p]
        _lib = handle
    return _lib


def _p(array):
    return array.ctypes.data_as(_f32p)


class ReferenceEngine:
    """The reference engine on the host cores (`threads` = its worker pool)."""

    SOLVERS = {"euler": 0, "heun": 1, "rk4": 2}
    SCHEDULERS = {"ddim": 0, "ddpm": 1}

    def __init__(self, path, threads: int = 0):
        self.lib = lib()
        self.handle = self.lib.fe_engine_load_with_threads(str(path).encode(), threads)
        if not self.handle:
            raise RuntimeError(self.lib.fe_engine_last_error().decode())

    @classmethod
    def from_weights(cls, weights, threads: int = 0):
        """Engine over a shared fe_weights store (fe_engine_create_from_weights)."""
        self = cls.__new__(cls)
        self.lib = lib()
        self.handle = self.lib.fe_engine_create_from_weights(weights, threads)
        if not self.handle:
            raise RuntimeError(self.lib.fe_engine_last_error().decode())
        return self

    def close(self):
        if self.handle:
            self.lib.fe_engine_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(f"reference status {rc}: {self.lib.fe_engine_last_error().decode()}")

    @property
    def action_dim(self):
        return self.lib.fe_engine_action_dim(self.handle)

    @property
    def horizon(self):
        return self.lib.fe_engine_action_horizon(self.handle)

    @property
    def condition_dim(self):
        return self.lib.fe_engine_condition_dim(self.handle)

    def metadata(self) -> dict:
        meta = _ModelMetadata()
        self._check(self.lib.fe_engine_model_metadata(self.handle, C.byref(meta)))
        return {name: (bytes(getattr(meta, name)) if name == "digest" else getattr(meta, name))
                for name, _ in _ModelMetadata._fields_}

    def sample_diffusion(self, condition, noise, steps, scheduler="ddim", seed=0):
        cond = np.ascontiguousarray(condition, np.float32)
        x = np.ascontiguousarray(noise, np.float32)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_sample_diffusion(
            self.handle, _p(cond), _p(x), steps, self.SCHEDULERS[scheduler], seed, _p(out)))
        return out

    def diffusion_denoise(self, condition, sample, timestep):
        cond = np.ascontiguousarray(condition, np.float32)
        x = np.ascontiguousarray(sample, np.float32)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_diffusion_denoise(self.handle, _p(cond), _p(x),
                                                         float(timestep), _p(out)))
        return out

    def sample_condition(self, condition, noise, steps, solver="euler"):
        cond = np.ascontiguousarray(condition, np.float32)
        x = np.ascontiguousarray(noise, np.float32)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_sample_condition(self.handle, _p(cond), _p(x), steps,
                                                        self.SOLVERS[solver], _p(out)))
        return out

    def sample(self, tokens, noise, steps, solver="euler"):
        toks = np.ascontiguousarray(tokens, np.int32)
        x = np.ascontiguousarray(noise, np.float32)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_sample(self.handle,
                                              toks.ctypes.data_as(C.POINTER(C.c_int32)),
                                              toks.size, _p(x), steps, self.SOLVERS[solver],
                                              _p(out)))
        return out

    def run(self, tokens, d_model):
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.empty((toks.size, d_model), np.float32)
        self._check(self.lib.fe_engine_run(self.handle, toks.ctypes.data_as(C.POINTER(C.c_int32)),
                                           toks.size, _p(out)))
        return out

    def step(self, token, d_model):
        out = np.empty(d_model, np.float32)
        self._check(self.lib.fe_engine_step(self.handle, int(token), _p(out)))
        return out

    def reset(self):
        self.lib.fe_engine_reset(self.handle)

    def export_decode_state(self) -> bytes:
        size = self.lib.fe_engine_decode_state_bytes(self.handle)
        buf = C.create_string_buffer(size)
        self._check(self.lib.fe_engine_export_decode_state(self.handle, buf, size))
        return buf.raw

    # SmolVLA action expert (engine.h:136-196); keys / values [layers][prefix][320]

    @staticmethod
    def _u8(array):
        return array.ctypes.data_as(C.POINTER(C.c_uint8))

    def smolvla_embed_suffix(self, noisy, timestep, width):
        x = np.ascontiguousarray(noisy, np.float32)
        chunk = x.shape[0]
        out = np.empty((chunk, width), np.float32)
        self._check(self.lib.fe_engine_smolvla_embed_suffix(self.handle, _p(x), chunk, float(timestep), _p(out)))
        return out

    def smolvla_run_expert(self, suffix, keys, values, mask):
        x = np.ascontiguousarray(suffix, np.float32)
        k, v = np.ascontiguousarray(keys, np.float32), np.ascontiguousarray(values, np.float32)
        m = np.ascontiguousarray(mask, np.uint8)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_smolvla_run_expert(self.handle, _p(x), x.shape[0], _p(k), _p(v), self._u8(m),
                                                          m.size, _p(out)))
        return out

    def smolvla_project_actions(self, hidden, action_dim):
        x = np.ascontiguousarray(hidden, np.float32)
        out = np.empty((x.shape[0], action_dim), np.float32)
        self._check(self.lib.fe_engine_smolvla_project_actions(self.handle, _p(x), x.shape[0], _p(out)))
        return out

    def smolvla_denoise(self, noisy, timestep, keys, values, mask):
        x = np.ascontiguousarray(noisy, np.float32)
        k, v = np.ascontiguousarray(keys, np.float32), np.ascontiguousarray(values, np.float32)
        m = np.ascontiguousarray(mask, np.uint8)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_smolvla_denoise(self.handle, _p(x), x.shape[0], float(timestep), _p(k), _p(v),
                                                       self._u8(m), m.size, _p(out)))
        return out

    def smolvla_sample(self, noise, steps, keys, values, mask):
        x = np.ascontiguousarray(noise, np.float32)
        k, v = np.ascontiguousarray(keys, np.float32), np.ascontiguousarray(values, np.float32)
        m = np.ascontiguousarray(mask, np.uint8)
        out = np.empty_like(x)
        self._check(self.lib.fe_engine_smolvla_sample(self.handle, _p(x), x.shape[0], steps, _p(k), _p(v),
                                                      self._u8(m), m.size, _p(out)))
        return out
