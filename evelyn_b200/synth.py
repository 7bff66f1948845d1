"""Seeded synthetic GGUF models (Qwen3 family) for tests and benchmarks.

The reference can read GGUF but has no encoder, so the quantisers live in
``csrc/synth_gguf.cpp`` (built into ``libevelyn_synth.so``). Weights are
N(0, stddev) from a counter-based generator, norms are 1.0, and the metadata
keys are those ``Model::load`` reads (src/runtime.rs:199-269).
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import os

import numpy as np

from . import _native

GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_BF16 = 0, 1, 8, 12, 13, 14, 30


def type_bytes(t: int, n: int) -> int:
    """gguf.rs:288-298."""
    return {GGML_F32: n * 4, GGML_F16: n * 2, GGML_BF16: n * 2, GGML_Q8_0: n // 32 * 34,
            GGML_Q4_K: n // 256 * 144, GGML_Q5_K: n // 256 * 176, GGML_Q6_K: n // 256 * 210}[t]


class _Spec(C.Structure):
    _fields_ = [
        ("arch", C.c_char * 32),
        ("layers", C.c_uint32), ("dim", C.c_uint32), ("ffn", C.c_uint32), ("heads", C.c_uint32),
        ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("vocab", C.c_uint32),
        ("rope_base", C.c_float), ("eps", C.c_float), ("stddev", C.c_float),
        ("type_attn_q", C.c_uint32), ("type_attn_k", C.c_uint32), ("type_attn_v", C.c_uint32),
        ("type_attn_output", C.c_uint32), ("type_ffn_gate", C.c_uint32), ("type_ffn_up", C.c_uint32),
        ("type_ffn_down", C.c_uint32), ("type_embed", C.c_uint32), ("type_output", C.c_uint32),
        ("qk_norm", C.c_uint32), ("tied_output", C.c_uint32), ("eos_token_id", C.c_uint32),
        ("seed", C.c_uint64), ("threads", C.c_int32),
        ("full_attention_interval", C.c_uint32), ("ssm_conv_kernel", C.c_uint32), ("ssm_state", C.c_uint32),
        ("ssm_groups", C.c_uint32), ("ssm_value_heads", C.c_uint32), ("ssm_inner", C.c_uint32),
        ("type_ssm", C.c_uint32), ("rope_dim", C.c_uint32), ("mrope_interleaved", C.c_uint32),
    ]


@dataclasses.dataclass
class ModelSpec:
    layers: int
    dim: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int = 128
    vocab: int = 151936
    rope_base: float = 1e6
    eps: float = 1e-6
    stddev: float = 0.02
    attn_q: int = GGML_Q4_K
    attn_k: int = GGML_Q4_K
    attn_v: int = GGML_Q6_K
    attn_output: int = GGML_Q4_K
    ffn_gate: int = GGML_Q4_K
    ffn_up: int = GGML_Q4_K
    ffn_down: int = GGML_Q6_K
    embed: int = GGML_Q8_0
    output: int = GGML_Q8_0
    qk_norm: bool = True
    tied_output: bool = False
    eos_token_id: int = 151645
    seed: int = 0
    arch: str = "qwen3"
    # arch "qwen35": gated-delta layers except every full_attention_interval-th
    full_attention_interval: int = 4
    ssm_conv_kernel: int = 4
    ssm_state: int = 64        # key_dim
    ssm_groups: int = 2        # key heads
    ssm_value_heads: int = 4
    ssm_inner: int = 256       # value_heads * value_dim
    ssm_type: int = GGML_Q8_0  # attn_qkv, attn_gate, ssm_alpha, ssm_beta, ssm_out
    rope_dim: int = 0          # 0: head_dim (key not written)
    mrope_interleaved: bool = False

    def with_types(self, t: int) -> "ModelSpec":
        return dataclasses.replace(self, attn_q=t, attn_k=t, attn_v=t, attn_output=t, ffn_gate=t, ffn_up=t,
                                   ffn_down=t, embed=t, output=t)

    def weight_bytes_per_token(self) -> int:
        """GGUF bytes of every matrix one decode step reads (embedding: one row), plus norms."""
        qw, kw = self.heads * self.head_dim, self.kv_heads * self.head_dim
        per_layer = (type_bytes(self.attn_q, self.dim * qw) + type_bytes(self.attn_k, self.dim * kw)
                     + type_bytes(self.attn_v, self.dim * kw) + type_bytes(self.attn_output, qw * self.dim)
                     + type_bytes(self.ffn_gate, self.dim * self.ffn) + type_bytes(self.ffn_up, self.dim * self.ffn)
                     + type_bytes(self.ffn_down, self.ffn * self.dim)
                     + 4 * (2 * self.dim + (2 * self.head_dim if self.qk_norm else 0)))
        head = type_bytes(self.embed if self.tied_output else self.output, self.dim * self.vocab)
        return self.layers * per_layer + head + type_bytes(self.embed, self.dim) + 4 * self.dim

    def kv_bytes_per_position(self, elem_bytes: int = 2) -> int:
        return 2 * self.layers * self.kv_heads * self.head_dim * elem_bytes


# The decoder shapes of the benchmark configurations.
def qwen35_tiny(**kw) -> ModelSpec:
    """A small Qwen3.5-style hybrid decoder (runtime.rs:455-630): gated-delta layers with
    one gated full-attention layer in every four, interleaved rotary positions."""
    base = dict(layers=4, dim=256, ffn=512, heads=4, kv_heads=2, head_dim=64, vocab=1024, arch="qwen35",
                mrope_interleaved=True)
    base.update(kw)
    return ModelSpec(**base)


def qwen35_hybrid_2b(**kw) -> ModelSpec:
    """A Qwen3.5-style hybrid decoder of about 2B parameters: 24 layers, every fourth full
    attention (8 Q / 2 KV heads x 256 with 64 rotary dimensions, gated query, interleaved
    rotary positions), the rest gated-delta layers (16 key heads x 128, 32 value heads x
    128, conv kernel 4), Q4_K_M-style weights."""
    base = dict(layers=24, dim=2048, ffn=6144, heads=8, kv_heads=2, head_dim=256, rope_dim=64, arch="qwen35",
                mrope_interleaved=True, full_attention_interval=4, ssm_conv_kernel=4, ssm_state=128,
                ssm_groups=16, ssm_value_heads=32, ssm_inner=4096, ssm_type=GGML_Q4_K)
    base.update(kw)
    return ModelSpec(**base)


def qwen3_0_6b(**kw) -> ModelSpec:
    """Qwen3-0.6B shape, every linear weight Q8_0."""
    return ModelSpec(layers=28, dim=1024, ffn=3072, heads=16, kv_heads=8, **kw).with_types(GGML_Q8_0)


def qwen3_8b(**kw) -> ModelSpec:
    """Qwen3-8B shape, Q4_K_M-style mix (attn_v / ffn_down Q6_K, embed / output Q8_0)."""
    return ModelSpec(layers=36, dim=4096, ffn=12288, heads=32, kv_heads=8, **kw)


def qwen3_32b(**kw) -> ModelSpec:
    """Qwen3-32B shape, Q4_K_M-style mix."""
    return ModelSpec(layers=64, dim=5120, ffn=25600, heads=64, kv_heads=8, **kw)


def tiny(**kw) -> ModelSpec:
    """A small decoder with the same structure, for parity tests."""
    base = dict(layers=2, dim=256, ffn=512, heads=4, kv_heads=2, head_dim=64, vocab=1024)
    base.update(kw)
    return ModelSpec(**base)


class GGUFImage:
    """A GGUF v3 file image in malloc'd host memory (freed on close/GC)."""

    def __init__(self, ptr: int, nbytes: int):
        self.ptr = ptr
        self.nbytes = nbytes

    def array(self) -> np.ndarray:
        return np.ctypeslib.as_array(C.cast(self.ptr, C.POINTER(C.c_uint8)), shape=(self.nbytes,))

    def write(self, path: str | os.PathLike):
        _check(_lib().evs_write_file(C.c_void_p(self.ptr), self.nbytes, os.fsencode(path)))

    def close(self):
        if getattr(self, "ptr", 0) and _L is not None:
            _L.evs_free(C.c_void_p(self.ptr))
        self.ptr = 0

    __del__ = close


_L = None


def _lib():
    global _L
    if _L is None:
        L = _native.load("libevelyn_synth.so")
        L.evs_last_error.restype = C.c_char_p
        L.evs_encode.argtypes = [C.c_uint32, C.POINTER(C.c_float), C.c_size_t, C.c_void_p, C.c_size_t]
        L.evs_f32_to_f16.restype = C.c_uint16
        L.evs_f32_to_f16.argtypes = [C.c_float]
        L.evs_build.argtypes = [C.POINTER(_Spec), C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
        L.evs_free.argtypes = [C.c_void_p]
        L.evs_write_file.argtypes = [C.c_void_p, C.c_size_t, C.c_char_p]
        _L = L
    return _L


def _check(rc: int):
    if rc != 0:
        raise RuntimeError(f"synth error {rc}: {_lib().evs_last_error().decode()}")


def build(spec: ModelSpec, threads: int = 0) -> GGUFImage:
    s = _Spec()
    s.arch = spec.arch.encode()
    for f in ("layers", "dim", "ffn", "heads", "kv_heads", "head_dim", "vocab", "rope_base", "eps", "stddev",
              "eos_token_id", "seed"):
        setattr(s, f, getattr(spec, f))
    s.type_attn_q, s.type_attn_k, s.type_attn_v = spec.attn_q, spec.attn_k, spec.attn_v
    s.type_attn_output, s.type_ffn_gate, s.type_ffn_up = spec.attn_output, spec.ffn_gate, spec.ffn_up
    s.type_ffn_down, s.type_embed, s.type_output = spec.ffn_down, spec.embed, spec.output
    s.qk_norm = int(spec.qk_norm)
    s.tied_output = int(spec.tied_output)
    s.threads = threads
    for f in ("full_attention_interval", "ssm_conv_kernel", "ssm_state", "ssm_groups", "ssm_value_heads",
              "ssm_inner", "rope_dim"):
        setattr(s, f, getattr(spec, f))
    s.type_ssm = spec.ssm_type
    s.mrope_interleaved = int(spec.mrope_interleaved)
    p = C.c_void_p()
    n = C.c_size_t()
    _check(_lib().evs_build(C.byref(s), C.byref(p), C.byref(n)))
    return GGUFImage(p.value, n.value)


def encode(ggml_type: int, x: np.ndarray) -> bytes:
    """Encode f32 values as one ggml type (whole blocks)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    nb = type_bytes(ggml_type, x.size)
    out = np.empty(nb, dtype=np.uint8)
    _check(_lib().evs_encode(ggml_type, x.ctypes.data_as(C.POINTER(C.c_float)), x.size, out.ctypes.data, nb))
    return out.tobytes()


def f32_to_f16_bits(v: float) -> int:
    return int(_lib().evs_f32_to_f16(v))
