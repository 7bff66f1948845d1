"""The routed-layer bridge driven from a GPU session (src/remote.rs:114-156 and
:247-271): layer 1 of a session goes through the engine's own AARNN client
(evl_remote_ffn_*) to a fake knowledge region on loopback that answers y = 2x, and the
session's logits must equal the oracle stepping the same tokens with that layer's FFN
replaced by 2 * ffn_input. A region that drops every request makes the layer fall back
to the device's dense FFN, counted by the backend's fallback counter, and the logits
then equal the plain dense session's. Failures are made on the host (the fake region),
never on the GPU."""
import numpy as np
import pytest

import evelyn_b200 as evl
from evelyn_b200 import synth
from oracle import oracle as orc
from tests.test_remote import FakeRegion

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3


def _tokens(n, vocab, seed):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def test_session_layer_served_by_remote_region():
    spec = synth.tiny(seed=9, layers=3)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0)
    r = orc.Model(img)
    srv = FakeRegion(["ok"] * 64)
    try:
        remote = evl.RemoteAarnnFfn(m, {1: f"127.0.0.1:{srv.port}"}, timeout=5.0)
        s, rs = evl.Session(m, max_ctx=64), orc.Session(r)
        worst = 0.0
        toks = _tokens(12, spec.vocab, seed=4)
        for tok in toks:
            got = s.step(tok, remote)
            want = rs.step(tok, lambda layer, x: 2 * x if layer == 1 else None)
            worst = max(worst, float(np.abs(got - want).max()))
        assert worst <= LOGIT_TOL, worst
        assert srv.requests == len(toks) and srv.connections == 1  # one persistent stream
        stats = remote.endpoint_stats()[1][1]
        assert stats["calls"] == len(toks) and stats["failures"] == 0
        assert remote.fallbacks == 0
    finally:
        srv.close()


def test_dropping_region_falls_back_to_device_dense_ffn():
    spec = synth.tiny(seed=19, layers=2)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0)
    srv = FakeRegion(["drop"] * 64)  # every attempt, including the reconnect, fails
    try:
        remote = evl.RemoteAarnnFfn(m, {0: f"127.0.0.1:{srv.port}"}, timeout=5.0)
        s, d = evl.Session(m, max_ctx=32), evl.Session(m, max_ctx=32)
        toks = _tokens(5, spec.vocab, seed=6)
        for tok in toks:
            assert np.abs(s.step(tok, remote) - d.step(tok)).max() <= 1e-4
        assert remote.fallbacks == len(toks)
        stats = remote.endpoint_stats()[0][1]
        assert stats["failures"] == len(toks) and stats["retries"] == len(toks)
    finally:
        srv.close()
