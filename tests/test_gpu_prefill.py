"""Batched prompt processing (evl_session_prefill) against the reference's way of
feeding a prompt -- one Session::step per token (src/bin/evelyn-generate.rs:69-80,
src/runtime.rs:773-808): every position's logits within the session tolerance of the
oracle, the session's position advanced by the prompt length, and the greedy decode
that follows identical to a session that stepped the prompt. Prompts of a length that
is not a multiple of the 32-row chunk exercise the padding rows; a prompt fed in two
calls checks that positions continue."""
import numpy as np
import pytest

import evelyn_b200 as evl
from evelyn_b200 import synth
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3


def _tokens(n, vocab, seed):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


@pytest.mark.parametrize("head_dim,heads,kv_heads,kv_f32", [(64, 4, 2, False), (128, 8, 2, False),
                                                            (128, 8, 2, True)])
def test_prefill_matches_stepwise_and_oracle(head_dim, heads, kv_heads, kv_f32):
    spec = synth.tiny(seed=51, head_dim=head_dim, heads=heads, kv_heads=kv_heads, layers=2)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0, kv_f32=kv_f32)
    r = orc.Model(img)
    prompt = _tokens(75, spec.vocab, seed=3)
    a, b, rs = evl.Session(m, max_ctx=160), evl.Session(m, max_ctx=160), orc.Session(r)
    got = a.prefill(prompt, logits=True)
    assert got.shape == (len(prompt), spec.vocab) and a.pos == len(prompt)
    worst = 0.0
    for i, tok in enumerate(prompt):
        want = rs.step(tok)
        worst = max(worst, float(np.abs(got[i] - want).max()))
        step = b.step(tok)
        assert np.abs(got[i] - step).max() <= LOGIT_TOL
    assert worst <= LOGIT_TOL, worst
    t = evl.argmax(got[-1])
    assert a.generate(t, 16) == b.generate(t, 16)
    assert a.pos == b.pos == len(prompt) + 16


def test_prefill_in_two_calls_continues_positions():
    spec = synth.tiny(seed=52, layers=2)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0)
    r = orc.Model(img)
    prompt = _tokens(70, spec.vocab, seed=5)
    s, rs = evl.Session(m, max_ctx=128), orc.Session(r)
    g1 = s.prefill(prompt[:40], logits=True)
    am = s.prefill(prompt[40:])  # argmax only
    assert s.pos == 70
    want = [rs.step(t) for t in prompt]
    assert max(float(np.abs(g1[i] - want[i]).max()) for i in range(40)) <= LOGIT_TOL
    assert am == [orc.argmax(w) for w in want[40:]]
    # the next step continues from position 70
    assert np.abs(s.step(3) - rs.step(3)).max() <= LOGIT_TOL


def test_prefill_errors():
    spec = synth.tiny(seed=53)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0)
    s = evl.Session(m, max_ctx=16)
    with pytest.raises(evl.EvelynError) as e:
        s.prefill([1, 2, spec.vocab])
    assert e.value.kind == "InvalidInput" and s.pos == 0
    with pytest.raises(evl.EvelynError) as e:
        s.prefill(list(range(17)))
    assert e.value.kind == "InvalidInput" and s.pos == 0
    assert s.prefill([]) == [] and s.pos == 0


def test_prefill_after_a_partial_chunk():
    """A prompt fed as 40 then 64 tokens: the second call's first chunk is full again
    after the first call ended on a padded one, so every row must map the session's
    pages again."""
    spec = synth.tiny(seed=54, layers=2)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0)
    r = orc.Model(img)
    prompt = _tokens(104, spec.vocab, seed=7)
    s, rs = evl.Session(m, max_ctx=160), orc.Session(r)
    g1 = s.prefill(prompt[:40], logits=True)
    g2 = s.prefill(prompt[40:], logits=True)
    want = [rs.step(t) for t in prompt]
    got = np.concatenate([g1, g2])
    assert max(float(np.abs(got[i] - want[i]).max()) for i in range(len(prompt))) <= LOGIT_TOL
    assert np.abs(s.step(9) - rs.step(9)).max() <= LOGIT_TOL


@pytest.mark.parametrize("kv_f32", [False, True])
def test_batch_prefill_per_sequence(kv_f32):
    """evl_batch_prefill: three sequences of one batch prefilled with prompts of
    different lengths (one of them in two calls), then decoded together: every
    prefill position and every batched step against the oracle run of that sequence,
    and the sequences' positions advanced independently."""
    spec = synth.tiny(seed=55, layers=2, head_dim=128, heads=8, kv_heads=2)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0, kv_f32=kv_f32)
    r = orc.Model(img)
    prompts = [_tokens(n, spec.vocab, seed=20 + n) for n in (45, 32, 70)]
    bat = evl.Batch(m, 3, max_ctx=96)
    ors = [orc.Session(r) for _ in prompts]
    worst = 0.0
    for i in (2, 0, 1):  # out of order: each call maps its own sequence's pages
        p = prompts[i]
        got = bat.prefill(i, p[:30], logits=True) if i == 2 else bat.prefill(i, p, logits=True)
        if i == 2:
            got = np.concatenate([got, bat.prefill(i, p[30:], logits=True)])
        for k, tok in enumerate(p):
            worst = max(worst, float(np.abs(got[k] - ors[i].step(tok)).max()))
        assert bat.pos(i) == len(p)
    assert worst <= LOGIT_TOL, worst
    toks = [5, 6, 7]
    for _ in range(8):
        lg = bat.step(toks)
        for i in range(3):
            worst = max(worst, float(np.abs(lg[i] - ors[i].step(toks[i])).max()))
        toks = [evl.argmax(lg[i]) for i in range(3)]
    assert worst <= LOGIT_TOL, worst
    assert [bat.pos(i) for i in range(3)] == [len(p) + 8 for p in prompts]
    with pytest.raises(evl.EvelynError) as e:
        bat.prefill(3, [1])
    assert e.value.kind == "InvalidInput"
