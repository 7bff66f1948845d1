"""The oracle, pinned before it is trusted.

1. The reference's own known-answer tests (tests/gguf.rs:20-81) and runtime unit
   tests (src/runtime.rs:816-841), restated against the oracle.
2. Random blocks against gguf-py's dequantiser (golden fixture, bit-for-bit).
3. Model-level semantics against HuggingFace transformers' Qwen3 in float32
   (golden fixture; see tests/golden/make_golden.py).
"""
import hashlib
import os

import numpy as np
import pytest

from evelyn_b200 import synth
from oracle import oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 8, 12, 13, 14, 30


def f16(v: float) -> bytes:
    """The f16 encoder of tests/gguf.rs:6-18 (exact for small powers of two and halves)."""
    bits = np.float32(v).view(np.uint32)
    sign = (bits >> 16) & 0x8000
    exp = int((bits >> 23) & 0xFF) - 127 + 15
    frac = (bits >> 13) & 0x3FF
    h = sign if v == 0.0 else sign | (exp << 10) | frac
    return int(h).to_bytes(2, "little")


# ------------------------------------------------------------------ tests/gguf.rs
def test_f16_and_bf16_round_trip():  # tests/gguf.rs:20-33
    for v in [0.0, 1.0, -2.5, 0.5, 65504.0]:
        assert orc.f16_to_f32(int.from_bytes(f16(v), "little")) == v
    sub = orc.f16_to_f32(0x0001)
    assert 0.0 < sub < 1e-7
    assert list(orc.dequantize(F16, f16(1.5), 1)) == [1.5]
    bf = (np.float32(-3.0).view(np.uint32) >> 16).astype(np.uint16)
    assert list(orc.dequantize(BF16, int(bf).to_bytes(2, "little"), 1)) == [-3.0]


def test_q8_0_block():  # tests/gguf.rs:35-43
    b = f16(0.5) + bytes(((i - 16) & 0xFF) for i in range(32))
    y = orc.dequantize(Q8_0, b, 32)
    assert y[0] == -8.0 and y[31] == 7.5


def test_q4_k_block():  # tests/gguf.rs:45-66
    sc = [0] * 12
    for j in range(4):
        sc[j] = 2
        sc[j + 4] = 1
    for j in range(8, 12):
        sc[j] = 2 | (1 << 4)
    b = f16(1.0) + f16(0.5) + bytes(sc) + bytes([0x53] * 128)
    y = orc.dequantize(Q4_K, b, 256)
    assert y[0] == 2.0 * 3.0 - 0.5
    assert y[32] == 2.0 * 5.0 - 0.5
    assert y[255] == 2.0 * 5.0 - 0.5


def test_q6_k_block():  # tests/gguf.rs:68-76
    b = bytes(128 + 64) + bytes([1] * 16) + f16(0.25)
    y = orc.dequantize(Q6_K, b, 256)
    assert np.all(y == -8.0)


def test_length_mismatch_is_an_error():  # tests/gguf.rs:78-81
    with pytest.raises(orc.OracleError) as e:
        orc.dequantize(Q8_0, bytes(34), 64)
    assert e.value.kind == "InvalidData"


def test_unsupported_type():  # gguf.rs:280-298
    with pytest.raises(orc.OracleError) as e:
        orc.dequantize(2, bytes(18), 32)  # Q4_0
    assert e.value.kind == "Unsupported"


# ------------------------------------------------------------------ runtime.rs unit tests
def test_token_validation():  # src/runtime.rs:816-826
    orc.validate_token_ids([0, 17, 99], 100)
    with pytest.raises(orc.OracleError) as e:
        orc.validate_token_ids([17, 100], 100)
    assert e.value.kind == "InvalidInput" and "tokenizer and GGUF match" in str(e.value)


def test_argmax_first_max_and_log_prob():  # src/runtime.rs:897-912
    v = np.array([1.0, 3.0, 3.0, -1.0], dtype=np.float32)
    assert orc.argmax(v) == 1
    assert orc.argmax(np.array([np.nan, 2.0, np.nan], dtype=np.float32)) == 1
    assert orc.argmax(np.full(3, -np.inf, dtype=np.float32)) == 0
    lp = orc.log_prob(v, 3)
    ref = -1.0 - np.log(np.exp(v - 3.0).sum()) - 3.0
    assert abs(lp - ref) < 1e-6


# ------------------------------------------------------------------ independent implementations
@pytest.mark.parametrize("t", [Q8_0, Q4_K, Q5_K, Q6_K])
def test_random_blocks_match_gguf_py(t):
    g = np.load(os.path.join(GOLDEN, "dequant_random.npz"))
    raw, want = g[f"raw_{t}"], g[f"y_{t}"]
    got = orc.dequantize(t, raw, want.size)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t", [Q8_0, Q4_K, Q5_K, Q6_K, F16, BF16, F32])
def test_synth_encoders_round_trip(t):
    rng = np.random.default_rng(t)
    x = (rng.standard_normal(256 * 16) * 0.02).astype(np.float32)
    y = orc.dequantize(t, synth.encode(t, x), x.size)
    bound = {Q8_0: 0.01, Q4_K: 0.1, Q5_K: 0.05, Q6_K: 0.03, F16: 1e-3, BF16: 1e-2, F32: 0.0}[t]
    assert np.abs(y - x).max() <= bound * np.abs(x).max()


def test_oracle_matches_hf_qwen3():
    g = np.load(os.path.join(GOLDEN, "tiny_qwen3_hf.npz"))
    img = synth.build(synth.tiny(seed=0))
    assert hashlib.sha256(img.array().tobytes()).hexdigest() == str(g["gguf_sha256"])
    m = orc.Model(img)
    s = orc.Session(m)
    worst = 0.0
    for i, tok in enumerate(g["tokens"]):
        worst = max(worst, float(np.abs(s.step(int(tok)) - g["logits"][i]).max()))
    assert worst < 1e-4, worst


def test_synth_is_deterministic_across_threads():
    a = synth.build(synth.tiny(seed=4), threads=1)
    b = synth.build(synth.tiny(seed=4), threads=8)
    assert np.array_equal(a.array(), b.array())


def test_model_load_errors():
    with pytest.raises(orc.OracleError) as e:
        orc.Model("/nonexistent.gguf")
    assert e.value.kind == "NotFound"
    with pytest.raises(orc.OracleError) as e:
        orc.Model(b"GGUX" + bytes(64))
    assert e.value.kind == "InvalidData"


def test_oracle_ffn_hook_and_dense_ffn():
    img = synth.build(synth.tiny(seed=1))
    m = orc.Model(img)
    a, b = orc.Session(m), orc.Session(m)
    calls = []

    def hook(layer, x):
        calls.append(layer)
        return m.dense_ffn(layer, x)

    for tok in [3, 9, 27]:
        assert np.array_equal(a.step(tok, hook), b.step(tok))
    assert calls == [0, 1] * 3


def _sample_py(logits, temperature, state):
    """src/server.rs:326-352 in plain Python (float32 weights summed in float64)."""
    if temperature <= np.finfo(np.float32).eps:
        return orc.argmax(logits), state
    lf = np.asarray(logits, dtype=np.float32)
    mx = np.float32(np.max(lf))
    w = np.exp((lf - mx) / np.float32(temperature)).astype(np.float64)
    total = 0.0
    for v in w:
        total += float(v)
    mask = (1 << 64) - 1
    x = state
    x ^= x >> 12
    x ^= (x << 25) & mask
    x ^= x >> 27
    unit = (((x * 0x2545F4914F6CDD1D) & mask) >> 11) / float(1 << 53)
    threshold = unit * total
    cum = 0.0
    for i, v in enumerate(w):
        cum += float(v)
        if cum >= threshold:
            return i, x
    return orc.argmax(logits), x


def test_sample_token_restatement():
    """The oracle's sample_token against a plain-Python restatement: same tokens, same
    xorshift64* states (exact integers), temperature 0 leaves the state alone."""
    rng = np.random.default_rng(0)
    for temperature in (0.0, 0.3, 1.0, 2.5):
        state = 12345
        for _ in range(20):
            logits = (rng.standard_normal(500) * 3).astype(np.float32)
            got = orc.sample_token(logits, temperature, state)
            assert got == _sample_py(logits, temperature, state)
            state = got[1]
