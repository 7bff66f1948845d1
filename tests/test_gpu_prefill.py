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
