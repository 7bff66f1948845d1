"""Python binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: tests, ``__graft_entry__.smoke()`` and the CPU-baseline
arm of ``bench.py`` use it as the checker / the timed reference algorithm. The
product (``evelyn_b200``) never imports it.

The oracle restates the reference's ``src/gguf.rs`` and ``src/runtime.rs`` in
C++ (see oracle.cpp for the line-by-line citations).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

ERROR_KINDS = {1: "InvalidInput", 2: "InvalidData", 3: "NotFound", 4: "Unsupported", 5: "Io"}


class OracleError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERROR_KINDS.get(code, code)}: {msg}")
        self.code = code
        self.kind = ERROR_KINDS.get(code, str(code))


class Config(C.Structure):
    _fields_ = [
        ("arch", C.c_char * 64),
        ("layers", C.c_uint64), ("dim", C.c_uint64), ("ffn", C.c_uint64), ("heads", C.c_uint64),
        ("kv_heads", C.c_uint64), ("head_dim", C.c_uint64), ("rope_dim", C.c_uint64), ("vocab", C.c_uint64),
        ("rope_base", C.c_float), ("eps", C.c_float),
        ("rope_interleaved", C.c_int32),
        ("eos_token_id", C.c_int64),
        ("full_attention_interval", C.c_uint64),
        ("ssm_conv_kernel", C.c_uint64), ("ssm_inner", C.c_uint64), ("ssm_state", C.c_uint64),
        ("ssm_groups", C.c_uint64), ("ssm_value_heads", C.c_uint64),
    ]


FFN_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_float), C.c_size_t, C.POINTER(C.c_float))


def build() -> str:
    """Compile liboracle.so with the committed Makefile (g++, no FP contraction)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        f = C.POINTER(C.c_float)
        L.orc_last_error.restype = C.c_char_p
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_get_threads.restype = C.c_int
        L.orc_type_bytes.restype = C.c_int64
        L.orc_type_bytes.argtypes = [C.c_uint32, C.c_uint64]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_dequantize.argtypes = [C.c_uint32, C.c_void_p, C.c_size_t, C.c_size_t, f]
        L.orc_model_load.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
        L.orc_model_load_memory.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]
        L.orc_model_free.argtypes = [C.c_void_p]
        L.orc_model_config.argtypes = [C.c_void_p, C.POINTER(Config)]
        L.orc_dense_ffn.argtypes = [C.c_void_p, C.c_size_t, f, f]
        L.orc_ffn_input.argtypes = [C.c_void_p, C.c_size_t, f, f]
        L.orc_matvec.argtypes = [C.c_void_p, C.c_char_p, f, C.c_size_t, f, C.c_size_t]
        L.orc_tensor_f32.argtypes = [C.c_void_p, C.c_char_p, f, C.c_size_t]
        L.orc_tensor_info.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64),
                                      C.POINTER(C.c_uint32)]
        L.orc_session_new.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
        L.orc_session_free.argtypes = [C.c_void_p]
        L.orc_session_pos.restype = C.c_uint64
        L.orc_session_pos.argtypes = [C.c_void_p]
        L.orc_session_step.argtypes = [C.c_void_p, C.c_uint32, FFN_FN, C.c_void_p, f]
        L.orc_session_fill_kv.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64]
        L.orc_validate_token_ids.argtypes = [C.POINTER(C.c_uint32), C.c_size_t, C.c_size_t]
        L.orc_gated_delta_step.restype = None
        L.orc_gated_delta_step.argtypes = [f, f, f, f, C.c_size_t, C.c_size_t, C.c_float, C.c_float, f]
        L.orc_rope_interleaved.restype = None
        L.orc_rope_interleaved.argtypes = [f, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float]
        L.orc_argmax.restype = C.c_uint32
        L.orc_argmax.argtypes = [f, C.c_size_t]
        L.orc_sample_token.restype = C.c_uint32
        L.orc_sample_token.argtypes = [f, C.c_size_t, C.c_float, C.POINTER(C.c_uint64)]
        L.orc_log_prob.restype = C.c_float
        L.orc_log_prob.argtypes = [f, C.c_size_t, C.c_uint32]
        _lib = L
    return _lib


def _check(rc: int):
    if rc != 0:
        raise OracleError(rc, lib().orc_last_error().decode(errors="replace"))


def _fp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def set_threads(n: int):
    lib().orc_set_threads(int(n))


def threads() -> int:
    return lib().orc_get_threads()


def type_bytes(t: int, n: int) -> int:
    v = lib().orc_type_bytes(t, n)
    if v < 0:
        raise OracleError(4, lib().orc_last_error().decode())
    return v


def f16_to_f32(h: int) -> float:
    return lib().orc_f16_to_f32(h)


def dequantize(t: int, raw: bytes | np.ndarray, n: int) -> np.ndarray:
    buf = np.frombuffer(bytes(raw), dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8)
    buf = np.ascontiguousarray(buf)
    out = np.empty(n, dtype=np.float32)
    _check(lib().orc_dequantize(t, buf.ctypes.data, buf.size, n, _fp(out)))
    return out


def validate_token_ids(ids, vocab: int):
    a = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
    _check(lib().orc_validate_token_ids(a.ctypes.data_as(C.POINTER(C.c_uint32)), a.size, vocab))


def gated_delta_step(state: np.ndarray, q, k, v, decay: float, beta: float) -> np.ndarray:
    """runtime.rs:493-528 on a [len(q), len(v)] f32 state, updated in place; returns the read-out."""
    q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
    assert state.dtype == np.float32 and state.flags.c_contiguous and state.size == q.size * v.size
    out = np.empty(v.size, dtype=np.float32)
    lib().orc_gated_delta_step(_fp(state), _fp(q), _fp(k), _fp(v), q.size, v.size, decay, beta, _fp(out))
    return out


def rope_interleaved(v: np.ndarray, heads: int, hd: int, rotary_dim: int, pos: int, base: float) -> np.ndarray:
    """runtime.rs:455-474 on a copy of v."""
    out = np.array(v, dtype=np.float32)
    lib().orc_rope_interleaved(_fp(out), heads, hd, rotary_dim, pos, base)
    return out


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, dtype=np.float32)
    return int(lib().orc_argmax(_fp(v), v.size))


def sample_token(logits: np.ndarray, temperature: float, state: int) -> tuple[int, int]:
    """server.rs:326-352; returns (token, new xorshift state)."""
    v = np.ascontiguousarray(logits, dtype=np.float32)
    st = C.c_uint64(state)
    tok = lib().orc_sample_token(_fp(v), v.size, temperature, C.byref(st))
    return int(tok), int(st.value)


def log_prob(logits: np.ndarray, target: int) -> float:
    v = np.ascontiguousarray(logits, dtype=np.float32)
    return float(lib().orc_log_prob(_fp(v), v.size, target))


def _buffer_ptr(source):
    if isinstance(source, np.ndarray):
        return source.ctypes.data, source.nbytes
    if hasattr(source, "ptr") and hasattr(source, "nbytes"):
        return source.ptr, source.nbytes
    arr = np.frombuffer(memoryview(source), dtype=np.uint8)
    return arr.ctypes.data, arr.nbytes


class Model:
    """Oracle Model (runtime.rs:184-425). Load from a path or a bytes-like GGUF image."""

    def __init__(self, source):
        h = C.c_void_p()
        if isinstance(source, (str, os.PathLike)):
            self._keep = None
            _check(lib().orc_model_load(os.fsencode(source), C.byref(h)))
        else:
            self._keep = source  # must outlive the model
            ptr, n = _buffer_ptr(source)
            _check(lib().orc_model_load_memory(ptr, n, C.byref(h)))
        self._h = h
        c = Config()
        lib().orc_model_config(h, C.byref(c))
        self.cfg = c

    def close(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.orc_model_free(self._h)
        self._h = None

    __del__ = close

    def dense_ffn(self, layer: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(self.cfg.dim, dtype=np.float32)
        _check(lib().orc_dense_ffn(self._h, layer, _fp(x), _fp(y)))
        return y

    def ffn_input(self, layer: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(self.cfg.dim, dtype=np.float32)
        _check(lib().orc_ffn_input(self._h, layer, _fp(x), _fp(y)))
        return y

    def tensor_info(self, name: str):
        t = C.c_uint32()
        dims = (C.c_uint64 * 4)()
        nd = C.c_uint32()
        _check(lib().orc_tensor_info(self._h, name.encode(), C.byref(t), dims, C.byref(nd)))
        return int(t.value), [int(dims[i]) for i in range(nd.value)]

    def tensor_f32(self, name: str) -> np.ndarray:
        _, dims = self.tensor_info(name)
        out = np.empty(int(np.prod(dims)), dtype=np.float32)
        _check(lib().orc_tensor_f32(self._h, name.encode(), _fp(out), out.size))
        return out

    def matvec(self, name: str, x: np.ndarray) -> np.ndarray:
        _, dims = self.tensor_info(name)
        rows = dims[1] if len(dims) > 1 else 1
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(rows, dtype=np.float32)
        _check(lib().orc_matvec(self._h, name.encode(), _fp(x), x.size, _fp(y), rows))
        return y


class Session:
    """Oracle Session (runtime.rs:634-808). `ffn` may be a callable (layer, x) -> y or None
    for the dense FFN; returning None from the callable also selects the dense FFN."""

    def __init__(self, model: Model):
        self.model = model
        h = C.c_void_p()
        _check(lib().orc_session_new(model._h, C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.orc_session_free(self._h)
        self._h = None

    __del__ = close

    @property
    def pos(self) -> int:
        return int(lib().orc_session_pos(self._h))

    def fill_kv(self, n: int, seed: int = 1):
        _check(lib().orc_session_fill_kv(self._h, n, seed))

    def step(self, token: int, ffn=None) -> np.ndarray:
        logits = np.empty(self.model.cfg.vocab, dtype=np.float32)
        if ffn is None:
            cb = FFN_FN()
        else:
            def _cb(ctx, layer, x, n, y):
                xa = np.ctypeslib.as_array(x, shape=(n,)).copy()
                out = ffn(int(layer), xa)
                if out is None:
                    return 1
                out = np.asarray(out, dtype=np.float32)
                if out.shape != (n,):
                    return 1
                np.ctypeslib.as_array(y, shape=(n,))[:] = out
                return 0
            cb = FFN_FN(_cb)
        _check(lib().orc_session_step(self._h, int(token) & 0xFFFFFFFF, cb, None, _fp(logits)))
        return logits
