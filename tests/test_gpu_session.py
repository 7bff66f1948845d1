"""Model-level parity of the device decode loop against the CPU oracle (a restatement
of src/runtime.rs:773-808): logits within max-abs 2e-3, greedy tokens identical,
perplexity within 0.5 %, plus the FfnBackend routing hook, batching and errors."""
import math

import numpy as np
import pytest

import evelyn_b200 as evl
from evelyn_b200 import synth
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3


def _models(spec, kv_f32=False):
    img = synth.build(spec)
    return img, evl.Model.load_memory(img, device=0, kv_f32=kv_f32), orc.Model(img)


def _tokens(n, vocab, seed=0):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


@pytest.mark.parametrize("kv_f32", [False, True])
@pytest.mark.parametrize("mix", ["q4k_mix", "q8_0", "q6k", "q5k", "f16", "bf16", "f32", "float_mix", "gate_up_mix"])
def test_step_logits_match_oracle(mix, kv_f32):
    """Unquantised (F16 / BF16 / F32) projections run the warp-per-row matvec; in
    "float_mix" the fused Q/K/V and gate/up launches hold an F16 matrix beside quantised
    ones, read through the exact dequantiser; "gate_up_mix" has a Q4_K gate beside a Q6_K up."""
    spec = synth.tiny(seed=11)
    if mix == "q8_0":
        spec = spec.with_types(synth.GGML_Q8_0)
    elif mix in ("q6k", "q5k"):
        spec = spec.with_types(synth.GGML_Q6_K if mix == "q6k" else synth.GGML_Q5_K)
        spec.embed = spec.output = synth.GGML_Q8_0
    elif mix in ("f16", "bf16", "f32"):
        spec = spec.with_types({"f16": synth.GGML_F16, "bf16": synth.GGML_BF16, "f32": synth.GGML_F32}[mix])
    elif mix == "float_mix":
        spec.attn_k = spec.ffn_up = synth.GGML_F16
        spec.attn_output = synth.GGML_BF16
        spec.output = synth.GGML_F32
    elif mix == "gate_up_mix":
        spec.ffn_up = synth.GGML_Q6_K
    img, m, r = _models(spec, kv_f32)
    s, rs = evl.Session(m, max_ctx=256), orc.Session(r)
    worst = 0.0
    for tok in _tokens(48, spec.vocab, seed=1):
        got, want = s.step(tok), rs.step(tok)
        worst = max(worst, float(np.abs(got - want).max()))
    assert s.pos == rs.pos == 48
    assert worst <= LOGIT_TOL, worst


def test_greedy_64_tokens_identical_and_ppl():
    spec = synth.tiny(seed=3, layers=3)
    img, m, r = _models(spec)
    s, rs = evl.Session(m, max_ctx=256), orc.Session(r)
    prompt = _tokens(32, spec.vocab, seed=2)
    nll_g = nll_o = 0.0
    for i, tok in enumerate(prompt):
        lg, lo = s.step(tok), rs.step(tok)
        if i + 1 < len(prompt):
            nll_g -= evl.log_prob(lg, prompt[i + 1])
            nll_o -= orc.log_prob(lo, prompt[i + 1])
    ppl_g, ppl_o = math.exp(nll_g / (len(prompt) - 1)), math.exp(nll_o / (len(prompt) - 1))
    assert abs(ppl_g / ppl_o - 1) < 0.005, (ppl_g, ppl_o)
    tg, to = evl.argmax(lg), orc.argmax(lo)
    out_g, out_o = [], []
    for _ in range(64):
        out_g.append(tg)
        out_o.append(to)
        tg, to = evl.argmax(s.step(tg)), orc.argmax(rs.step(to))
    assert out_g == out_o


def test_generate_matches_stepwise_argmax():
    spec = synth.tiny(seed=5)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0)
    a, b = evl.Session(m, max_ctx=128), evl.Session(m, max_ctx=128)
    toks = a.generate(17, 40)
    ref, t = [], 17
    for _ in range(40):
        t = b.step(t, logits=False)
        ref.append(t)
    assert toks == ref
    assert a.pos == b.pos == 40


class _OracleFfn(evl.FfnBackend):
    """Serves chosen layers from the oracle's dense FFN on the host (a stand-in AARNN region)."""

    def __init__(self, oracle_model, layers):
        self.o = oracle_model
        self.routed_layers = layers
        self.calls = []

    def ffn(self, layer, x):
        self.calls.append(layer)
        return self.o.dense_ffn(layer, x)


def test_ffn_routing_hook_matches_dense():
    spec = synth.tiny(seed=9, layers=3)
    img, m, r = _models(spec)
    hook = _OracleFfn(r, [1])
    s_hook, s_dense = evl.Session(m, max_ctx=64), evl.Session(m, max_ctx=64)
    for tok in _tokens(12, spec.vocab, seed=4):
        a, b = s_hook.step(tok, hook), s_dense.step(tok, evl.DenseFfn(m))
        assert np.abs(a - b).max() <= LOGIT_TOL
    assert hook.calls == [1] * 12


def test_capture_ffn_records_ffn_input():
    spec = synth.tiny(seed=9)
    img, m, r = _models(spec)
    cap = evl.CaptureFfn(m, 1)
    s, rs = evl.Session(m, max_ctx=64), orc.Session(r)
    captured = []
    for tok in _tokens(5, spec.vocab, seed=6):
        s.step(tok, cap)
        rs.step(tok, lambda layer, x: (captured.append(x) if layer == 1 else None) or None)
    assert len(cap.captured) == 5
    for g, w in zip(cap.captured, captured):
        assert np.abs(g - w).max() <= 1e-3


def test_failing_hook_falls_back_to_dense():
    spec = synth.tiny(seed=9)
    img, m, r = _models(spec)

    class Broken(evl.FfnBackend):
        routed_layers = [0]

        def ffn(self, layer, x):
            raise ConnectionError("region down")

    s, d = evl.Session(m, max_ctx=32), evl.Session(m, max_ctx=32)
    for tok in _tokens(4, spec.vocab, seed=8):
        assert np.abs(s.step(tok, Broken()) - d.step(tok)).max() <= LOGIT_TOL
    assert s.fallbacks == 4


@pytest.mark.parametrize("B,gemm,attn", [(3, "1", {}), (32, "1", {}), (3, "0", {}), (32, "1", {"EVELYN_ATTN_MMA": "0"}),
                                         (5, "1", {"EVELYN_ATTN_RING": "2"})])
def test_batch_matches_independent_sessions(B, gemm, attn, monkeypatch):
    """A Batch step (tensor-core products for 2..32 sequences, or one matvec per
    sequence with EVELYN_BATCH_GEMM=0; tensor-core cluster attention, its pages streamed
    through a 2-page ring, or the split attention kernels with EVELYN_ATTN_MMA=0)
    against independent sessions and the oracle."""
    monkeypatch.setenv("EVELYN_BATCH_GEMM", gemm)
    for k, v in attn.items():
        monkeypatch.setenv(k, v)
    spec = synth.tiny(seed=13)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0)
    r = orc.Model(img)
    batch = evl.Batch(m, B, max_ctx=64)
    sessions = [evl.Session(m, max_ctx=64) for _ in range(min(B, 4))]
    oracles = [orc.Session(r) for _ in range(min(B, 2))]
    rng = np.random.default_rng(0)
    worst = 0.0
    for _ in range(40 if attn else 10):
        toks = rng.integers(0, spec.vocab, B)
        got = batch.step(toks)
        for i, s in enumerate(sessions):
            assert np.abs(got[i] - s.step(int(toks[i]))).max() <= LOGIT_TOL
        for i, o in enumerate(oracles):
            worst = max(worst, float(np.abs(got[i] - o.step(int(toks[i]))).max()))
    assert worst <= LOGIT_TOL, worst


@pytest.mark.parametrize("stages", ["2", "4"])
def test_batch_attention_ring_stages(stages, monkeypatch):
    """Long splits streamed through a multi-stage ring (one split per sequence, 8-page
    ring: stages of 4 or 2 pages, so the stages wrap many times) against independent
    sessions and the oracle."""
    monkeypatch.setenv("EVELYN_ATTN_SPLITS", "1")
    monkeypatch.setenv("EVELYN_ATTN_RING", "8")
    monkeypatch.setenv("EVELYN_ATTN_STAGES", stages)
    spec = synth.tiny(seed=17, layers=2)
    img, m, r = _models(spec)
    batch = evl.Batch(m, 2, max_ctx=320)
    for k in ("EVELYN_ATTN_SPLITS", "EVELYN_ATTN_RING", "EVELYN_ATTN_STAGES"):
        monkeypatch.delenv(k)
    s, o = evl.Session(m, max_ctx=320), orc.Session(r)
    rng = np.random.default_rng(5)
    worst = 0.0
    for _ in range(300):
        toks = rng.integers(0, spec.vocab, 2)
        got = batch.step(toks)
        assert np.abs(got[0] - s.step(int(toks[0]))).max() <= LOGIT_TOL
        worst = max(worst, float(np.abs(got[1] - o.step(int(toks[1]))).max()))
    assert worst <= LOGIT_TOL, worst


def test_model_level_apis_match_oracle():
    spec = synth.tiny(seed=21)
    img, m, r = _models(spec)
    rng = np.random.default_rng(1)
    x = rng.standard_normal(spec.dim).astype(np.float32)
    assert np.abs(m.ffn_input(0, x) - r.ffn_input(0, x)).max() <= 1e-5
    xn = r.ffn_input(1, x)
    y, yo = m.dense_ffn(1, xn), r.dense_ffn(1, xn)
    assert np.abs(y - yo).max() <= 1e-4 * max(1.0, float(np.abs(yo).max()))
    for name in ("token_embd.weight", "blk.0.attn_q.weight", "blk.1.attn_v.weight", "blk.1.ffn_down.weight",
                 "output.weight", "blk.0.attn_norm.weight"):
        want = r.tensor_f32(name)
        got = m.dequantize(name, want.size)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name
    w = r.tensor_f32("blk.0.ffn_gate.weight").reshape(spec.ffn, spec.dim).astype(np.float64)
    assert np.abs(m.matvec("blk.0.ffn_gate.weight", x, spec.ffn) - w @ x).max() <= 1e-4


def test_tied_lm_head():
    spec = synth.tiny(seed=2, tied_output=True)
    img, m, r = _models(spec)
    s, rs = evl.Session(m, max_ctx=32), orc.Session(r)
    for tok in _tokens(6, spec.vocab, seed=3):
        assert np.abs(s.step(tok) - rs.step(tok)).max() <= LOGIT_TOL


def test_token_and_context_errors():
    spec = synth.tiny(seed=1)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0)
    s = evl.Session(m, max_ctx=4)
    with pytest.raises(evl.EvelynError) as e:
        s.step(spec.vocab)
    assert e.value.kind == "InvalidInput" and "tokenizer and GGUF match" in str(e.value)
    assert s.pos == 0
    for t in range(4):
        s.step(t)
    with pytest.raises(evl.EvelynError) as e:
        s.step(0)
    assert e.value.kind == "InvalidInput"
    # the session survives an error
    s2 = evl.Session(m, max_ctx=8)
    s2.step(1)
    assert s2.pos == 1


def test_load_errors():
    with pytest.raises(evl.EvelynError) as e:
        evl.Model.load("/nonexistent/model.gguf", device=0)
    assert e.value.kind == "NotFound"
    with pytest.raises(evl.EvelynError) as e:
        evl.Model.load_memory(b"GGUX" + b"\0" * 64, device=0)
    assert e.value.kind == "InvalidData"


@pytest.mark.parametrize("ring,mma", [(2, "0"), (4, "0"), (2, "1"), (16, "1")])
def test_cluster_attention_streamed_pages(monkeypatch, ring, mma):
    """Single-sequence attention with its KV pages streamed through a small shared ring
    (many chunks per split), on the scalar loop or the tensor cores, against the
    unfused three-kernel path and the oracle."""
    spec = synth.tiny(seed=23, layers=2)
    img, m, r = _models(spec)
    toks = _tokens(150, spec.vocab, seed=9)
    monkeypatch.setenv("EVELYN_ATTN_RING", str(ring))
    monkeypatch.setenv("EVELYN_ATTN_MMA", mma)
    s1 = evl.Session(m, max_ctx=256)
    out1 = [s1.step(t) for t in toks]
    monkeypatch.delenv("EVELYN_ATTN_RING")
    monkeypatch.delenv("EVELYN_ATTN_MMA")
    monkeypatch.setenv("EVELYN_FUSED_ATTN", "0")
    s2 = evl.Session(m, max_ctx=256)
    out2 = [s2.step(t) for t in toks]
    assert s1.kernels_per_step < s2.kernels_per_step  # one attention launch per layer vs three
    assert max(float(np.abs(a - b).max()) for a, b in zip(out1, out2)) <= 1e-4
    rs = orc.Session(r)
    worst = max(float(np.abs(a - rs.step(t)).max()) for a, t in zip(out1, toks))
    assert worst <= LOGIT_TOL, worst


def test_step_kernel_matches_launch_sequence(monkeypatch):
    """The persistent whole-step kernel (every layer and the LM head in one launch,
    phases handing vectors on as tagged words) against the per-kernel launch sequence
    on the same model and tokens: same logits within the attention's summation-order
    tolerance, same greedy tokens, and far fewer launches; then against the oracle."""
    spec = synth.tiny(seed=21, layers=3)
    img, m, r = _models(spec)
    toks = _tokens(150, spec.vocab, seed=4)
    monkeypatch.setenv("EVELYN_STEP_KERNEL", "1")
    s1 = evl.Session(m, max_ctx=256)
    out1 = [s1.step(t) for t in toks]
    monkeypatch.setenv("EVELYN_STEP_KERNEL", "0")
    s2 = evl.Session(m, max_ctx=256)
    out2 = [s2.step(t) for t in toks]
    assert s1.kernels_per_step == 4 < s2.kernels_per_step
    assert max(float(np.abs(a - b).max()) for a, b in zip(out1, out2)) <= 1e-4
    g1 = s1.generate(evl.argmax(out1[-1]), 24)
    g2 = s2.generate(evl.argmax(out2[-1]), 24)
    assert list(g1) == list(g2)
    rs = orc.Session(r)  # and the oracle
    worst = max(float(np.abs(a - rs.step(t)).max()) for a, t in zip(out1, toks))
    assert worst <= LOGIT_TOL, worst


@pytest.mark.parametrize("heads,kv_heads,kv_f32", [(4, 2, False), (8, 1, False), (4, 4, True), (8, 2, True)])
def test_step_kernel_groups_and_kv_types(heads, kv_heads, kv_f32, monkeypatch):
    """The persistent step kernel at GQA groups 2, 8, 1, 4 (head_dim 128) with f16 and
    f32 KV pages, past several attention chunks per split, against the oracle."""
    monkeypatch.setenv("EVELYN_STEP_KERNEL", "1")
    spec = synth.tiny(seed=40 + heads + kv_heads, head_dim=128, heads=heads, kv_heads=kv_heads, layers=2)
    img, m, r = _models(spec, kv_f32=kv_f32)
    s, rs = evl.Session(m, max_ctx=700), orc.Session(r)
    worst = 0.0
    for i, tok in enumerate(_tokens(650, spec.vocab, seed=heads)):
        want = rs.step(tok)
        if i % 13 == 0 or i > 640:
            got = s.step(tok)
            assert s.kernels_per_step == 4
            worst = max(worst, float(np.abs(got - want).max()))
        else:
            s.step(tok, logits=False)
    assert worst <= LOGIT_TOL, worst


@pytest.mark.parametrize("kv_f32", [False, True])
def test_head_dim_256_session_and_batch(kv_f32):
    """256-wide heads (GQA group 8) take the split attention kernels, one sequence and a
    batch of three (tensor-core products, paged attention per sequence)."""
    spec = synth.tiny(seed=41, head_dim=256, heads=8, kv_heads=1, layers=2)
    img, m, r = _models(spec, kv_f32)
    s, rs = evl.Session(m, max_ctx=128), orc.Session(r)
    worst = 0.0
    for tok in _tokens(40, spec.vocab, seed=3):
        worst = max(worst, float(np.abs(s.step(tok) - rs.step(tok)).max()))
    assert worst <= LOGIT_TOL, worst
    n = 3
    bt = evl.Batch(m, n, max_ctx=64)
    sessions = [orc.Session(r) for _ in range(n)]
    toks = [_tokens(20, spec.vocab, seed=50 + i) for i in range(n)]
    worst = 0.0
    for t in range(20):
        got = bt.step([toks[i][t] for i in range(n)])
        for i in range(n):
            worst = max(worst, float(np.abs(got[i] - sessions[i].step(toks[i][t])).max()))
    assert worst <= LOGIT_TOL, worst
