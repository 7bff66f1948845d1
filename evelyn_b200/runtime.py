"""Python mirror of Evelyn's runtime API over the engine's C ABI (include/evelyn.h).

Names, argument meanings and errors follow the reference (src/runtime.rs, src/remote.rs):

    model = Model.load(path)                     # Model::load          runtime.rs:199
    s = Session(model)                           # Session::new         runtime.rs:643
    logits = s.step(token, DenseFfn(model))      # Session::step        runtime.rs:773
    argmax(logits), log_prob(logits, target)     #                      runtime.rs:897, :908
    model.dense_ffn(layer, x), model.ffn_input(layer, x)                runtime.rs:409, :422

FfnBackend (runtime.rs:138) keeps the per-layer routing hook: DenseFfn runs every
FFN on the device; CaptureFfn records one layer's inputs (remote.rs:29-45);
RemoteAarnnFfn sends chosen layers to AARNN regions over TCP (remote.rs:163-272);
any object with ``ffn(layer, x) -> y`` works too. Errors raise EvelynError with
the io::ErrorKind name of the reference's error.

Every call runs the CUDA engine; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import os
from typing import Iterable, Optional

import numpy as np

from . import _native

EVL_FFN_DENSE = 1
_KINDS = {1: "InvalidInput", 2: "InvalidData", 3: "NotFound", 4: "Unsupported", 5: "Io", 6: "Cuda",
          7: "OutOfMemory", 8: "Nccl", 9: "TimedOut"}


class EvelynError(RuntimeError):
    """An engine error; ``kind`` is the io::ErrorKind-style name, ``code`` the evl_status."""

    def __init__(self, code: int, msg: str):
        self.code = code
        self.kind = _KINDS.get(code, str(code))
        super().__init__(f"{self.kind}: {msg}")


class _Config(C.Structure):
    _fields_ = [
        ("arch", C.c_char * 64),
        ("layers", C.c_uint64), ("dim", C.c_uint64), ("ffn", C.c_uint64), ("heads", C.c_uint64),
        ("kv_heads", C.c_uint64), ("head_dim", C.c_uint64), ("rope_dim", C.c_uint64), ("vocab", C.c_uint64),
        ("rope_base", C.c_float), ("eps", C.c_float), ("rope_interleaved", C.c_int32), ("eos_token_id", C.c_int64),
    ]


class _SsmConfig(C.Structure):
    _fields_ = [
        ("has_ssm", C.c_int32), ("delta_layers", C.c_uint32), ("full_attention_interval", C.c_uint64),
        ("conv_kernel", C.c_uint64), ("inner", C.c_uint64), ("state", C.c_uint64), ("groups", C.c_uint64),
        ("value_heads", C.c_uint64),
    ]


class _Options(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32), ("device", C.c_int32), ("tp_rank", C.c_int32), ("tp_size", C.c_int32),
        ("nccl_id", C.c_uint8 * 128), ("kv_f32", C.c_uint32), ("reserved", C.c_uint32 * 7),
    ]


_FFN_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_float), C.c_size_t, C.POINTER(C.c_float))


class _Backend(C.Structure):
    _fields_ = [("ffn", _FFN_FN), ("ctx", C.c_void_p), ("routed", C.POINTER(C.c_uint8)), ("routed_len", C.c_size_t),
                ("fallbacks", C.POINTER(C.c_uint64))]


class _EndpointStats(C.Structure):
    _fields_ = [("calls", C.c_uint64), ("failures", C.c_uint64), ("retries", C.c_uint64), ("total_ns", C.c_uint64),
                ("max_ns", C.c_uint64)]


class _TpShard(C.Structure):
    _fields_ = [("q_rows", C.c_uint64 * 2), ("kv_rows", C.c_uint64 * 2), ("ffn_rows", C.c_uint64 * 2),
                ("vocab_rows", C.c_uint64 * 2)]


@dataclasses.dataclass(frozen=True)
class Config:
    """runtime.rs:93-110 (dense-attention fields)."""
    arch: str
    layers: int
    dim: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int
    rope_dim: int
    vocab: int
    rope_base: float
    eps: float
    rope_interleaved: bool
    eos_token_id: Optional[int]


_L = None
LIB_NAME = "libevelyn_b200.so"

# every symbol include/evelyn.h declares, with its ctypes signature
_P = C.c_void_p
_F = C.POINTER(C.c_float)
_U32P = C.POINTER(C.c_uint32)
SIGNATURES = {
    "evl_last_error": (C.c_char_p, []),
    "evl_abi_version": (C.c_uint32, []),
    "evl_model_options_init": (None, [C.POINTER(_Options)]),
    "evl_validate_token_ids": (C.c_int, [_U32P, C.c_size_t, C.c_size_t]),
    "evl_argmax": (C.c_uint32, [_F, C.c_size_t]),
    "evl_log_prob": (C.c_float, [_F, C.c_size_t, C.c_uint32]),
    "evl_tp_unique_id": (C.c_int, [C.POINTER(C.c_uint8)]),
    "evl_tp_shard_plan": (C.c_int, [C.POINTER(_Config), C.c_int32, C.c_int32, C.POINTER(_TpShard)]),
    "evl_model_load": (C.c_int, [C.c_char_p, C.POINTER(_Options), C.POINTER(_P)]),
    "evl_model_load_memory": (C.c_int, [_P, C.c_size_t, C.POINTER(_Options), C.POINTER(_P)]),
    "evl_model_free": (None, [_P]),
    "evl_model_config": (C.c_int, [_P, C.POINTER(_Config)]),
    "evl_model_dense_ffn": (C.c_int, [_P, C.c_size_t, _F, _F]),
    "evl_model_ffn_input": (C.c_int, [_P, C.c_size_t, _F, _F]),
    "evl_model_dequantize": (C.c_int, [_P, C.c_char_p, _F, C.c_size_t]),
    "evl_model_matvec": (C.c_int, [_P, C.c_char_p, _F, C.c_size_t, _F, C.c_size_t]),
    "evl_model_weight_bytes": (C.c_uint64, [_P]),
    "evl_model_ssm_config": (C.c_int, [_P, C.POINTER(_SsmConfig)]),
    "evl_session_new": (C.c_int, [_P, C.c_uint32, C.POINTER(_P)]),
    "evl_session_free": (None, [_P]),
    "evl_session_pos": (C.c_uint64, [_P]),
    "evl_session_step": (C.c_int, [_P, C.c_uint32, C.POINTER(_Backend), _F, _U32P]),
    "evl_session_generate": (C.c_int, [_P, C.c_uint32, C.c_uint32, _U32P]),
    "evl_session_prefill": (C.c_int, [_P, _U32P, C.c_size_t, _F, _U32P]),
    "evl_session_sample": (C.c_int, [_P, C.c_float, C.POINTER(C.c_uint64), _U32P]),
    "evl_batch_sample": (C.c_int, [_P, C.c_float, C.POINTER(C.c_uint64), _U32P]),
    "evl_batch_prefill": (C.c_int, [_P, C.c_uint32, _U32P, C.c_size_t, _F, _U32P]),
    "evl_session_stream": (_P, [_P]),
    "evl_session_kernels_per_step": (C.c_uint32, [_P]),
    "evl_session_notes": (C.c_char_p, [_P]),
    "evl_batch_new": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.POINTER(_P)]),
    "evl_batch_free": (None, [_P]),
    "evl_batch_pos": (C.c_uint64, [_P, C.c_uint32]),
    "evl_batch_step": (C.c_int, [_P, _U32P, _F, _U32P]),
    "evl_batch_stream": (_P, [_P]),
    "evl_dequantize_raw": (C.c_int, [C.c_uint32, _P, C.c_size_t, _P, _P]),
    "evl_qmatrix_create": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, _P, C.c_int, C.POINTER(_P)]),
    "evl_qmatrix_free": (None, [_P]),
    "evl_qmatrix_bytes": (C.c_uint64, [_P]),
    "evl_qmatrix_matvec": (C.c_int, [_P, _P, _P, _P]),
    "evl_qmatrix_dequantize": (C.c_int, [_P, _P, _P]),
    "evl_qmatrix_matmul": (C.c_int, [_P, _P, C.c_uint32, _P, _P]),
    "evl_attention_decode": (C.c_int, [_P, _P, _P, _P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                       _P, _P]),
    "evl_attention_workspace_bytes": (C.c_size_t, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
    "evl_attention_decode_ws": (C.c_int, [_P, _P, _P, _P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                          C.c_uint32, _P, _P, C.c_size_t, _P]),
    "evl_attention_decode_noalloc": (C.c_int, [_P, _P, _P, _P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                               C.c_uint32, _P, _P]),
    "evl_remote_ffn_new": (C.c_int, [_P, C.c_size_t, C.POINTER(C.c_size_t), C.POINTER(C.c_char_p), C.c_uint32,
                                     C.POINTER(_P)]),
    "evl_remote_ffn_free": (None, [_P]),
    "evl_remote_ffn_backend": (C.c_int, [_P, C.POINTER(_Backend)]),
    "evl_remote_ffn_fallbacks": (C.c_uint64, [_P]),
    "evl_remote_ffn_stats": (C.c_int, [_P, C.c_size_t, C.POINTER(_EndpointStats)]),
}


def _prefer_wheel_nccl():
    """Point the engine's run-time NCCL lookup at the NCCL wheel PyTorch uses, when it is
    installed, so the engine and torch never load two NCCL builds under one soname."""
    if os.environ.get("EVELYN_NCCL_LIBRARY"):
        return
    try:
        import nvidia
        for base in list(getattr(nvidia, "__path__", [])):
            cand = os.path.join(base, "nccl", "lib", "libnccl.so.2")
            if os.path.exists(cand):
                os.environ["EVELYN_NCCL_LIBRARY"] = cand
                return
    except ImportError:
        pass


def lib():
    """The loaded engine library (raises NativeLibraryMissing when it is not built)."""
    global _L
    if _L is None:
        _prefer_wheel_nccl()
        L = _native.load(LIB_NAME)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _L = L
    return _L


def check(rc: int):
    if rc != 0:
        raise EvelynError(rc, lib().evl_last_error().decode(errors="replace"))


_check = check


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_F)


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


# ---------------------------------------------------------------- free functions
def validate_token_ids(tokens: Iterable[int], vocab: int) -> None:
    """runtime.rs:125-135: InvalidInput if any id >= vocab."""
    a = np.ascontiguousarray(np.asarray(list(tokens), dtype=np.uint32))
    _check(lib().evl_validate_token_ids(a.ctypes.data_as(_U32P), a.size, vocab))


def argmax(logits: np.ndarray) -> int:
    """runtime.rs:897-905: the first maximum (strict '>' from f32::MIN)."""
    v = _f32(logits)
    return int(lib().evl_argmax(_fp(v), v.size))


def log_prob(logits: np.ndarray, target: int) -> float:
    """runtime.rs:908-912."""
    v = _f32(logits)
    return float(lib().evl_log_prob(_fp(v), v.size, int(target)))


def tp_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    _check(lib().evl_tp_unique_id(buf))
    return bytes(buf)


def _options(device, tp_rank, tp_size, nccl_id, kv_f32) -> _Options:
    o = _Options()
    lib().evl_model_options_init(C.byref(o))
    o.device = -1 if device is None else int(device)
    o.tp_rank, o.tp_size = int(tp_rank), int(tp_size)
    if nccl_id is not None:
        C.memmove(o.nccl_id, bytes(nccl_id), 128)
    o.kv_f32 = int(bool(kv_f32))
    return o


# ---------------------------------------------------------------- model
class Model:
    """runtime.rs Model: quantised weights resident (repacked) in HBM."""

    def __init__(self, handle, opts: _Options):
        self._h = handle
        c = _Config()
        _check(lib().evl_model_config(handle, C.byref(c)))
        self.cfg = Config(arch=c.arch.decode(), layers=c.layers, dim=c.dim, ffn=c.ffn, heads=c.heads,
                          kv_heads=c.kv_heads, head_dim=c.head_dim, rope_dim=c.rope_dim, vocab=c.vocab,
                          rope_base=c.rope_base, eps=c.eps, rope_interleaved=bool(c.rope_interleaved),
                          eos_token_id=None if c.eos_token_id < 0 else int(c.eos_token_id))
        self.tp_rank, self.tp_size = opts.tp_rank, opts.tp_size

    @classmethod
    def load(cls, path: str | os.PathLike, device: Optional[int] = None, tp_rank: int = 0, tp_size: int = 1,
             nccl_id: Optional[bytes] = None, kv_f32: bool = False) -> "Model":
        o = _options(device, tp_rank, tp_size, nccl_id, kv_f32)
        h = C.c_void_p()
        _check(lib().evl_model_load(os.fsencode(path), C.byref(o), C.byref(h)))
        return cls(h, o)

    @classmethod
    def load_memory(cls, image, device: Optional[int] = None, tp_rank: int = 0, tp_size: int = 1,
                    nccl_id: Optional[bytes] = None, kv_f32: bool = False) -> "Model":
        """Load from a GGUF image in host memory (bytes, numpy array, or an object with .ptr/.nbytes)."""
        o = _options(device, tp_rank, tp_size, nccl_id, kv_f32)
        if hasattr(image, "ptr") and hasattr(image, "nbytes"):
            ptr, n = image.ptr, image.nbytes
        else:
            arr = np.frombuffer(memoryview(image), dtype=np.uint8)
            ptr, n = arr.ctypes.data, arr.nbytes
        h = C.c_void_p()
        _check(lib().evl_model_load_memory(C.c_void_p(ptr), n, C.byref(o), C.byref(h)))
        return cls(h, o)

    def close(self):
        if getattr(self, "_h", None) and _L is not None:
            _L.evl_model_free(self._h)
        self._h = None

    __del__ = close

    @property
    def handle(self):
        return self._h

    @property
    def weight_bytes(self) -> int:
        return int(lib().evl_model_weight_bytes(self._h))

    @property
    def ssm_config(self) -> dict:
        """Config::full_attention_interval and SsmConfig (runtime.rs:106-120), with the
        number of gated-delta layers; has_ssm False for models other than qwen35."""
        c = _SsmConfig()
        _check(lib().evl_model_ssm_config(self._h, C.byref(c)))
        return {"has_ssm": bool(c.has_ssm), "delta_layers": c.delta_layers,
                "full_attention_interval": c.full_attention_interval, "conv_kernel": c.conv_kernel,
                "inner": c.inner, "state": c.state, "groups": c.groups, "value_heads": c.value_heads}

    def dense_ffn(self, layer: int, x: np.ndarray) -> np.ndarray:
        """runtime.rs:409-418, on the device."""
        x = _f32(x)
        y = np.empty(self.cfg.dim, dtype=np.float32)
        _check(lib().evl_model_dense_ffn(self._h, layer, _fp(x), _fp(y)))
        return y

    def ffn_input(self, layer: int, x: np.ndarray) -> np.ndarray:
        """runtime.rs:422-424."""
        x = _f32(x)
        y = np.empty(self.cfg.dim, dtype=np.float32)
        _check(lib().evl_model_ffn_input(self._h, layer, _fp(x), _fp(y)))
        return y

    def dequantize(self, tensor: str, n: int) -> np.ndarray:
        """Exact device dequantisation of a tensor (this rank's shard), gguf.rs:199."""
        out = np.empty(n, dtype=np.float32)
        _check(lib().evl_model_dequantize(self._h, tensor.encode(), _fp(out), n))
        return out

    def matvec(self, tensor: str, x: np.ndarray, rows: int) -> np.ndarray:
        """QMatrix::matvec of one model matrix (runtime.rs:72-88)."""
        x = _f32(x)
        y = np.empty(rows, dtype=np.float32)
        _check(lib().evl_model_matvec(self._h, tensor.encode(), _fp(x), x.size, _fp(y), rows))
        return y


# ---------------------------------------------------------------- FFN backends
class FfnBackend:
    """runtime.rs:138-140. Subclasses implement ``ffn(layer, x) -> y``; returning None
    asks the engine to run the dense FFN for that layer on the device.
    ``routed_layers`` limits which layers cross to the host (None: all)."""

    routed_layers: Optional[Iterable[int]] = None

    def ffn(self, layer: int, x: np.ndarray) -> Optional[np.ndarray]:
        raise NotImplementedError


class DenseFfn(FfnBackend):
    """runtime.rs:428-434: the model's own dense FFN on every layer (stays on the device)."""

    def __init__(self, model: Model):
        self.model = model

    def ffn(self, layer, x):
        return self.model.dense_ffn(layer, x)


class CaptureFfn(FfnBackend):
    """remote.rs:29-45: dense FFN everywhere, recording the normalised FFN input of one layer."""

    def __init__(self, model: Model, layer: int):
        self.model = model
        self.layer = layer
        self.captured: list[np.ndarray] = []
        self.routed_layers = [layer]

    def ffn(self, layer, x):
        if layer == self.layer:
            self.captured.append(np.array(x, copy=True))
        return None  # dense on the device


class RemoteAarnnFfn(FfnBackend):
    """remote.rs:163-272: layers -> "host:port" AARNN regions, one reconnect, dense fallback.
    Runs natively (the engine's TCP client); the host crossing happens only on routed layers."""

    def __init__(self, model: Model, layers: dict[int, str], timeout: float = 900.0):
        self.model = model
        items = sorted(layers.items())
        ids = (C.c_size_t * max(1, len(items)))(*[k for k, _ in items])
        self._addrs = [a.encode() for _, a in items]
        addrs = (C.c_char_p * max(1, len(items)))(*self._addrs)
        h = C.c_void_p()
        _check(lib().evl_remote_ffn_new(model._h, len(items), ids, addrs, int(timeout * 1000), C.byref(h)))
        self._h = h
        self.routed_layers = [k for k, _ in items]
        self._backend = _Backend()
        _check(lib().evl_remote_ffn_backend(h, C.byref(self._backend)))

    @property
    def fallbacks(self) -> int:
        return int(lib().evl_remote_ffn_fallbacks(self._h))

    def endpoint_stats(self) -> dict:
        out = {}
        for layer, addr in zip(self.routed_layers, self._addrs):
            st = _EndpointStats()
            _check(lib().evl_remote_ffn_stats(self._h, layer, C.byref(st)))
            out[layer] = (addr.decode(), dict(calls=st.calls, failures=st.failures, retries=st.retries,
                                              total_ns=st.total_ns, max_ns=st.max_ns))
        return out

    def ffn(self, layer, x):  # not used: the native backend is passed straight through
        raise RuntimeError("RemoteAarnnFfn is served natively by the engine")

    def close(self):
        if getattr(self, "_h", None) and _L is not None:
            _L.evl_remote_ffn_free(self._h)
        self._h = None

    __del__ = close


def _make_backend(ffn: Optional[FfnBackend], n_layers: int):
    """Translate a Python FfnBackend into the C hook (None: dense on the device)."""
    if ffn is None or type(ffn) is DenseFfn:
        return None, None
    if isinstance(ffn, RemoteAarnnFfn):
        return ffn._backend, None

    def cb(ctx, layer, x, n, y):
        try:
            out = ffn.ffn(int(layer), np.ctypeslib.as_array(x, shape=(n,)).copy())
            if out is None:
                return EVL_FFN_DENSE
            out = np.asarray(out, dtype=np.float32)
            if out.shape != (n,):
                return 2
            np.ctypeslib.as_array(y, shape=(n,))[:] = out
            return 0
        except Exception:  # an exception in the hook becomes a dense fallback
            return 2

    keep = _FFN_FN(cb)
    b = _Backend()
    b.ffn = keep
    routed = None
    if ffn.routed_layers is not None:
        routed = (C.c_uint8 * n_layers)()
        for layer in ffn.routed_layers:
            if 0 <= layer < n_layers:
                routed[layer] = 1
        b.routed = C.cast(routed, C.POINTER(C.c_uint8))
        b.routed_len = n_layers
    fallbacks = C.c_uint64(0)
    b.fallbacks = C.pointer(fallbacks)
    return b, (keep, routed, fallbacks)


# ---------------------------------------------------------------- sessions
class Session:
    """runtime.rs:634-808: one sequence with a paged KV cache on the device."""

    def __init__(self, model: Model, max_ctx: int = 4096):
        self.model = model
        h = C.c_void_p()
        _check(lib().evl_session_new(model._h, int(max_ctx), C.byref(h)))
        self._h = h
        self.fallbacks = 0  # hook failures that fell back to the dense FFN

    def close(self):
        if getattr(self, "_h", None) and _L is not None:
            _L.evl_session_free(self._h)
        self._h = None

    __del__ = close

    @property
    def handle(self):
        return self._h

    @property
    def pos(self) -> int:
        return int(lib().evl_session_pos(self._h))

    @property
    def stream(self) -> int:
        return int(lib().evl_session_stream(self._h) or 0)

    @property
    def kernels_per_step(self) -> int:
        return int(lib().evl_session_kernels_per_step(self._h))

    @property
    def notes(self) -> str:
        """Why the opt-in persistent step kernel is not used, if it was asked for."""
        return (lib().evl_session_notes(self._h) or b"").decode()

    def step(self, token: int, ffn: Optional[FfnBackend] = None, logits: bool = True):
        """Feed one token; returns next-token logits (a new array), or the argmax when logits=False."""
        backend, keep = _make_backend(ffn, self.model.cfg.layers)
        am = C.c_uint32()
        out = np.empty(self.model.cfg.vocab, dtype=np.float32) if logits else None
        _check(lib().evl_session_step(self._h, int(token) & 0xFFFFFFFF, C.byref(backend) if backend else None,
                                      _fp(out) if logits else None, C.byref(am)))
        if keep is not None and keep[2] is not None:
            self.fallbacks += int(keep[2].value)
        return out if logits else int(am.value)

    def sample(self, temperature: float, state: int) -> tuple[int, int]:
        """server.rs:326-352 on the device from the last step's logits: returns (token,
        new xorshift64* state); temperature <= FLT_EPSILON is the greedy pick."""
        st = C.c_uint64(state)
        tok = C.c_uint32()
        _check(lib().evl_session_sample(self._h, float(temperature), C.byref(st), C.byref(tok)))
        return int(tok.value), int(st.value)

    def prefill(self, tokens, logits: bool = False):
        """Feed a prompt in batched steps (as len(tokens) step calls would); returns the
        per-position logits [n][vocab] when logits=True, else the per-position argmax."""
        t = np.ascontiguousarray(np.asarray(list(tokens), dtype=np.uint32))
        am = np.empty(max(1, t.size), dtype=np.uint32)
        out = np.empty((t.size, self.model.cfg.vocab), dtype=np.float32) if logits else None
        _check(lib().evl_session_prefill(self._h, t.ctypes.data_as(_U32P), t.size,
                                         _fp(out) if logits else None, am.ctypes.data_as(_U32P)))
        return out if logits else [int(v) for v in am[:t.size]]

    def generate(self, token: int, n: int) -> list[int]:
        """Greedy decode on the device: feeds `token`, then each step's argmax (n steps)."""
        out = np.empty(max(1, n), dtype=np.uint32)
        _check(lib().evl_session_generate(self._h, int(token), int(n), out.ctypes.data_as(_U32P)))
        return [int(t) for t in out[:n]]


class Batch:
    """n independent sequences decoded together (one token each per step)."""

    def __init__(self, model: Model, n_seqs: int, max_ctx: int = 4096):
        self.model = model
        self.n = n_seqs
        h = C.c_void_p()
        _check(lib().evl_batch_new(model._h, int(n_seqs), int(max_ctx), C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None) and _L is not None:
            _L.evl_batch_free(self._h)
        self._h = None

    __del__ = close

    def pos(self, seq: int) -> int:
        return int(lib().evl_batch_pos(self._h, seq))

    @property
    def stream(self) -> int:
        return int(lib().evl_batch_stream(self._h) or 0)

    def step(self, tokens, logits: bool = True):
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        if t.size != self.n:
            raise EvelynError(1, f"expected {self.n} tokens, got {t.size}")
        am = np.empty(self.n, dtype=np.uint32)
        out = np.empty((self.n, self.model.cfg.vocab), dtype=np.float32) if logits else None
        _check(lib().evl_batch_step(self._h, t.ctypes.data_as(_U32P), _fp(out) if logits else None,
                                    am.ctypes.data_as(_U32P)))
        return out if logits else am

    def prefill(self, seq: int, tokens, logits: bool = False):
        """Session.prefill for sequence `seq` of the batch: its prompt in batched steps;
        per-position logits [n][vocab] when logits=True, else the per-position argmax."""
        t = np.ascontiguousarray(np.asarray(list(tokens), dtype=np.uint32))
        am = np.empty(max(1, t.size), dtype=np.uint32)
        out = np.empty((t.size, self.model.cfg.vocab), dtype=np.float32) if logits else None
        _check(lib().evl_batch_prefill(self._h, int(seq), t.ctypes.data_as(_U32P), t.size,
                                       _fp(out) if logits else None, am.ctypes.data_as(_U32P)))
        return out if logits else [int(v) for v in am[:t.size]]

    def sample(self, temperature: float, states):
        """Session.sample for every sequence: returns (tokens, new states)."""
        st = np.ascontiguousarray(np.asarray(states, dtype=np.uint64))
        if st.size != self.n:
            raise EvelynError(1, f"expected {self.n} states, got {st.size}")
        tok = np.empty(self.n, dtype=np.uint32)
        _check(lib().evl_batch_sample(self._h, float(temperature), st.ctypes.data_as(C.POINTER(C.c_uint64)),
                                      tok.ctypes.data_as(_U32P)))
        return [int(v) for v in tok], [int(v) for v in st]
