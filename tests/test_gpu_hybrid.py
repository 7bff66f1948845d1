"""Qwen3.5 hybrid decoding on the device (src/runtime.rs:455-630, 684-695, 753-761)
against the CPU oracle: gated-delta layers (projections as matvec launches, the conv /
delta-rule / norm-and-gate kernel of gated_delta.cu) and the gated full-attention layer,
logits within max-abs 2e-3 at every step, 64 identical greedy tokens and PPL within
0.5 %, for one sequence, a batch and the FFN routing hook."""
import math

import numpy as np
import pytest

import evelyn_b200 as evl
from evelyn_b200 import synth
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3


def _tokens(n, vocab, seed):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


@pytest.mark.parametrize("kv_f32", [False, True])
@pytest.mark.parametrize("variant", ["q8_0", "q4_k", "neox_partial_rope", "kernel2", "alpha_beta_apart",
                                     "one_cta_per_head", "head_dim_256", "f16_ssm", "q5_k_ssm", "all_full_attention"])
def test_hybrid_step_logits_match_oracle(variant, kv_f32, monkeypatch):
    """alpha_beta_apart: ssm_alpha and ssm_beta as two matrices with a launch of their
    own (EVELYN_DELTA_STACK=0) instead of stacked into the projections' launch;
    one_cta_per_head: the gated-delta kernel without the cluster split of the value
    columns (EVELYN_DELTA_SLICES=0)."""
    kw = {}
    if variant == "alpha_beta_apart":
        monkeypatch.setenv("EVELYN_DELTA_STACK", "0")
    if variant == "one_cta_per_head":
        monkeypatch.setenv("EVELYN_DELTA_SLICES", "0")
    if variant == "head_dim_256":  # Qwen3.5's own full-attention heads: 256 wide, 64 rotary dims
        kw = dict(head_dim=256, rope_dim=64)
    if variant == "f16_ssm":  # unquantised projections: the warp-per-row matvec, three segments
        kw = dict(ssm_type=synth.GGML_F16)
    if variant == "q5_k_ssm":
        kw = dict(ssm_type=synth.GGML_Q5_K)
    if variant == "all_full_attention":  # interval 1: every layer gated full attention
        kw = dict(full_attention_interval=1)
    if variant == "q4_k":
        kw = dict(ssm_type=synth.GGML_Q4_K)
    elif variant == "neox_partial_rope":
        kw = dict(mrope_interleaved=False, rope_dim=32)
    elif variant == "kernel2":  # a 2-tap conv, 3 value heads over 1 key head, interval 2
        kw = dict(ssm_conv_kernel=2, ssm_groups=1, ssm_value_heads=3, ssm_inner=192, ssm_state=64,
                  full_attention_interval=2)
    spec = synth.qwen35_tiny(seed=17, **kw)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0, kv_f32=kv_f32)
    sc = m.ssm_config
    assert sc["has_ssm"] and sc["value_heads"] == spec.ssm_value_heads
    assert sc["delta_layers"] == sum((i + 1) % spec.full_attention_interval != 0 for i in range(spec.layers))
    r = orc.Model(img)
    s, rs = evl.Session(m, max_ctx=128), orc.Session(r)
    worst = 0.0
    for tok in _tokens(40, spec.vocab, seed=1):
        got, want = s.step(tok), rs.step(tok)
        worst = max(worst, float(np.abs(got - want).max()))
    assert s.pos == rs.pos == 40
    assert worst <= LOGIT_TOL, worst


def test_hybrid_greedy_64_and_ppl():
    spec = synth.qwen35_tiny(seed=8, layers=8)
    img = synth.build(spec)
    m, r = evl.Model.load_memory(img, device=0), orc.Model(img)
    s, rs = evl.Session(m, max_ctx=128), orc.Session(r)
    prompt = _tokens(24, spec.vocab, seed=4)
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


@pytest.mark.parametrize("kv_f32", [False, True])
def test_hybrid_batch_matches_oracle_per_sequence(kv_f32):
    """Three sequences with their own recurrent states and positions (the batch runs the
    matvecs per sequence; the gated-delta kernel takes the batch as its grid's y). f16
    pages take the cluster attention, f32 pages the split kernels: both apply the query
    gate as they write their output."""
    spec = synth.qwen35_tiny(seed=12)
    img = synth.build(spec)
    m, r = evl.Model.load_memory(img, device=0, kv_f32=kv_f32), orc.Model(img)
    n = 3
    bt = evl.Batch(m, n, max_ctx=64)
    sessions = [orc.Session(r) for _ in range(n)]
    toks = [_tokens(20, spec.vocab, seed=30 + i) for i in range(n)]
    worst = 0.0
    for t in range(20):
        got = bt.step([toks[i][t] for i in range(n)])
        for i in range(n):
            worst = max(worst, float(np.abs(got[i] - sessions[i].step(toks[i][t])).max()))
    assert worst <= LOGIT_TOL, worst


def test_hybrid_routed_ffn_and_unsupported_paths():
    """The FFN hook sees the hybrid layers like any other (a host FFN from the oracle
    gives the oracle's logits); a single session's prefill runs one step per prompt
    token; batch prefill and tensor parallelism answer Unsupported for the hybrid model."""
    spec = synth.qwen35_tiny(seed=3)
    img = synth.build(spec)
    m, r = evl.Model.load_memory(img, device=0), orc.Model(img)
    s, rs = evl.Session(m, max_ctx=64), orc.Session(r)
    seen = []

    class HostFfn(evl.FfnBackend):
        def ffn(self, layer, x):
            seen.append(layer)
            return r.dense_ffn(layer, x)

    ffn = HostFfn()
    worst = 0.0
    for tok in _tokens(6, spec.vocab, seed=9):
        worst = max(worst, float(np.abs(s.step(tok, ffn=ffn) - rs.step(tok)).max()))
    assert worst <= LOGIT_TOL, worst
    assert seen == list(range(spec.layers)) * 6
    # prefill: one step per prompt token for a single session (the reference's own loop),
    # refused for a batch of several sequences
    p, po = evl.Session(m, max_ctx=64), orc.Session(r)
    prompt = _tokens(8, spec.vocab, seed=1)
    rows = p.prefill(prompt, logits=True)
    worst = max(float(np.abs(rows[i] - po.step(t)).max()) for i, t in enumerate(prompt))
    worst = max(worst, float(np.abs(p.step(5) - po.step(5)).max()))
    assert p.pos == po.pos == 9 and worst <= LOGIT_TOL, worst
    bt = evl.Batch(m, 2, max_ctx=64)
    with pytest.raises(evl.EvelynError) as e:
        bt.prefill(0, prompt)
    assert e.value.kind == "Unsupported"
    # tensor parallelism is refused at load, before any communicator is made
    with pytest.raises(evl.EvelynError) as e:
        evl.Model.load_memory(img, device=0, tp_rank=0, tp_size=2, nccl_id=evl.tp_unique_id())
    assert e.value.kind == "Unsupported"
