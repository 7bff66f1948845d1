"""Helpers for GPU tests: device buffers come from torch (plumbing only); every
computation under test goes through the engine's C ABI."""
from __future__ import annotations

import ctypes as C

import numpy as np


def torch():
    import torch as _t
    return _t


def to_dev(a: np.ndarray):
    t = torch()
    return t.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


def empty_f32(n: int):
    t = torch()
    return t.empty(n, dtype=t.float32, device="cuda:0")


def ptr(t) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def sync():
    torch().cuda.synchronize()


def random_blocks(ggml_type: int, nblocks: int, rng: np.random.Generator) -> bytes:
    """Random raw GGUF blocks: arbitrary quant bytes with finite, moderate f16 scales."""
    from evelyn_b200 import synth
    bb = {synth.GGML_Q8_0: 34, synth.GGML_Q4_K: 144, synth.GGML_Q5_K: 176, synth.GGML_Q6_K: 210}[ggml_type]
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    def f16(vals):
        return np.asarray(vals, dtype=np.float16).view(np.uint8).reshape(-1, 2)
    if ggml_type == synth.GGML_Q8_0:
        raw[:, 0:2] = f16(rng.uniform(-0.05, 0.05, nblocks))
    elif ggml_type in (synth.GGML_Q4_K, synth.GGML_Q5_K):
        raw[:, 0:2] = f16(rng.uniform(0, 0.01, nblocks))
        raw[:, 2:4] = f16(rng.uniform(0, 0.01, nblocks))
    else:  # Q6_K: d at 208
        raw[:, 208:210] = f16(rng.uniform(-0.01, 0.01, nblocks))
    # a few subnormal and zero scales to exercise f16_to_f32's edge cases
    if nblocks >= 4:
        off = 208 if ggml_type == synth.GGML_Q6_K else 0
        raw[0, off:off + 2] = [0x01, 0x00]   # smallest subnormal
        raw[1, off:off + 2] = [0xff, 0x03]   # largest subnormal
        raw[2, off:off + 2] = [0x00, 0x80]   # -0
    return raw.tobytes()
