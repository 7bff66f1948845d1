"""Parity at the benchmarked shapes (src/runtime.rs:773-808 through the C ABI against
the CPU oracle):

* the Qwen3-0.6B-shape (28 layers, all Q8_0) and Qwen3-8B-shape (36 layers, Q4_K_M
  mix) synthetic models: a 16-token random prompt fed to both, teacher-forced
  perplexity over it, then 64 greedy steps from each side's own argmax -- logits
  within max-abs 2e-3 at every step (f32 KV, the reference's precision; f16 KV pages
  within 2e-2), identical greedy tokens, PPL within 0.5 % (the protocol of
  src/bin/evelyn-generate.rs:69-86);
* head_dim 128 sessions with GQA groups 1, 2, 4 and 8 run past 1200 positions, so the
  single-sequence cluster attention streams its 8 splits through the page ring at the
  benchmark's head size (tensor-core loop over f16 pages, scalar loop over f16 and f32
  pages; the default ring and a 2-page ring), and the persistent step kernel's
  attention phase runs its splits over many chunks;
* the matvec paths only the big shapes reach: the LM-head shape 151936x4096 Q8_0
  (more row blocks per CTA than partial buffers: rotating buffers, last-warp
  reduction) and 5120x25600 Q6_K (rows longer than 12288 values: quarter staging).
"""
import ctypes as C
import gc
import json
import math
import os

import numpy as np
import pytest

import evelyn_b200 as evl
from evelyn_b200 import runtime, synth
from oracle import oracle as orc
from tests import gpu_util as gu

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3


def _tokens(n, vocab, seed):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def _top2_margin(logits):
    top = np.partition(logits, -2)[-2:]
    return float(top[1] - top[0])


def _oracle_protocol(img, spec, prompt, steps):
    """The oracle's side of the protocol: logits at every prompt position and greedy
    step, its teacher-forced NLL and greedy tokens."""
    r = orc.Model(img)
    rs = orc.Session(r)
    logits, nll = [], 0.0
    for i, tok in enumerate(prompt):
        logits.append(rs.step(tok))
        if i + 1 < len(prompt):
            nll -= orc.log_prob(logits[-1], prompt[i + 1])
    greedy = []
    for _ in range(steps):
        greedy.append(orc.argmax(logits[-1]))
        logits.append(rs.step(greedy[-1]))
    return logits, math.exp(nll / (len(prompt) - 1)), greedy


def _engine_protocol(img, spec, prompt, steps, want, kv_f32):
    """The same protocol on the device (greedy from its own argmax); returns the worst
    logit difference from the oracle's `want`, its PPL and greedy tokens."""
    m = evl.Model.load_memory(img, device=0, kv_f32=kv_f32)
    s = evl.Session(m, max_ctx=len(prompt) + steps + 8)
    worst, nll = 0.0, 0.0
    for i, tok in enumerate(prompt):
        lg = s.step(tok)
        worst = max(worst, float(np.abs(lg - want[i]).max()))
        if i + 1 < len(prompt):
            nll -= evl.log_prob(lg, prompt[i + 1])
    greedy = []
    for j in range(steps):
        greedy.append(evl.argmax(lg))
        lg = s.step(greedy[-1])
        worst = max(worst, float(np.abs(lg - want[len(prompt) + j]).max()))
    del s, m
    gc.collect()
    return worst, math.exp(nll / (len(prompt) - 1)), greedy


# f16 KV pages round every cached K and V element to 11 bits, which the f32 reference
# (src/runtime.rs:721-722 keeps f32 rows) does not: at the 8B shape that moves logits by
# about 1e-2 (measured 0.011 worst over 28 steps) while the greedy tokens stay the same.
# The strict bar applies to the reference's own KV precision.
F16_KV_LOGIT_TOL = 2e-2


@pytest.mark.slow
@pytest.mark.parametrize("shape", ["qwen3_0_6b", "qwen3_8b"])
def test_benchmark_shape_generate_matches_oracle(shape):
    """16 prompt tokens (teacher-forced PPL) then 64 greedy steps, the oracle once and
    the engine with f32 KV pages and with f16 KV pages."""
    spec = getattr(synth, shape)(seed=0)
    img = synth.build(spec)
    prompt, steps = _tokens(16, spec.vocab, 0), 64
    want, ppl_o, greedy_o = _oracle_protocol(img, spec, prompt, steps)
    margin = min(_top2_margin(w) for w in want[len(prompt) - 1:])
    rows = []
    for kv_f32, tol in ((True, LOGIT_TOL), (False, F16_KV_LOGIT_TOL)):
        worst, ppl_g, greedy_g = _engine_protocol(img, spec, prompt, steps, want, kv_f32)
        rows.append({"shape": shape, "kv": "f32" if kv_f32 else "f16", "max_abs": worst, "tol": tol, "ppl": ppl_g,
                     "ppl_oracle": ppl_o, "greedy_equal": greedy_g == greedy_o, "greedy_steps": steps,
                     "min_top2_margin": margin})
        assert worst <= tol, (kv_f32, worst)
        assert abs(ppl_g / ppl_o - 1) < 0.005, (kv_f32, ppl_g, ppl_o)
        assert greedy_g == greedy_o, (kv_f32, greedy_g, greedy_o, margin)
    rdir = os.environ.get("EVELYN_PARITY_RESULT_DIR")
    if rdir:  # the measured figures, for a summary beside the test run
        with open(os.path.join(rdir, f"parity_{shape}.json"), "w") as f:
            f.write(json.dumps(rows) + "\n")


@pytest.mark.parametrize("heads,kv_heads", [(4, 4), (4, 2), (8, 2), (8, 1)])
@pytest.mark.parametrize("path,ring", [("cluster", None), ("cluster", "2"), ("stages4", "8"), ("scalar", None),
                                       ("f32", None), ("f32", "2"), ("step", None)])
def test_hd128_attention_long_context(heads, kv_heads, path, ring, monkeypatch):
    """GQA group 1 / 2 / 4 / 8 at head_dim 128 (the 0.6B, 8B and 32B groups are 2, 4
    and 8) past 1200 positions, through the launch sequence's cluster attention -- the
    tensor-core loop over f16 pages, the scalar loop over f16 pages (EVELYN_ATTN_MMA=0)
    and over f32 pages, each with the default ring and some with a 2-page ring, and the
    double-buffered 4-stage ring (8 pages) -- and
    through the persistent step kernel: every 25th step's logits against the oracle,
    and greedy agreement."""
    monkeypatch.setenv("EVELYN_STEP_KERNEL", "1" if path == "step" else "0")
    if path == "scalar":
        monkeypatch.setenv("EVELYN_ATTN_MMA", "0")
    if path == "stages4":  # double-buffered: two warp groups, each alternating between two stages
        monkeypatch.setenv("EVELYN_ATTN_STAGES", "4")
    if ring:
        monkeypatch.setenv("EVELYN_ATTN_RING", ring)
    spec = synth.tiny(seed=31 + heads + kv_heads, head_dim=128, heads=heads, kv_heads=kv_heads, layers=2)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=0, kv_f32=path == "f32")
    r = orc.Model(img)
    s, rs = evl.Session(m, max_ctx=1280), orc.Session(r)
    toks = _tokens(1240, spec.vocab, seed=heads * 10 + kv_heads)
    worst = 0.0
    for i, tok in enumerate(toks):
        want = rs.step(tok)
        if i % 25 == 0 or i >= len(toks) - 4:
            got = s.step(tok)
            worst = max(worst, float(np.abs(got - want).max()))
            assert evl.argmax(got) == orc.argmax(want) or _top2_margin(want) < 2 * LOGIT_TOL
        else:
            s.step(tok, logits=False)
    assert s.pos == rs.pos == len(toks)
    assert worst <= LOGIT_TOL, worst


def _big_matvec_case(t, rows, cols, seed):
    rng = np.random.default_rng(seed)
    block = 32 if t == synth.GGML_Q8_0 else 256
    raw = gu.random_blocks(t, rows * cols // block, rng)
    x = rng.standard_normal(cols).astype(np.float32)
    # reference in row chunks: exact dequantisation by the oracle, product in float64
    rb = synth.type_bytes(t, cols)
    want = np.empty(rows)
    scale = np.empty(rows)
    xd = x.astype(np.float64)
    step = 4096
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        w = orc.dequantize(t, raw[r0 * rb:r1 * rb], (r1 - r0) * cols).reshape(r1 - r0, cols).astype(np.float64)
        want[r0:r1] = w @ xd
        scale[r0:r1] = np.abs(w) @ np.abs(xd)
    return raw, x, want, scale


@pytest.mark.slow
@pytest.mark.parametrize("t,rows,cols", [(synth.GGML_Q8_0, 151936, 4096), (synth.GGML_Q6_K, 5120, 25600),
                                         (synth.GGML_Q4_K, 25600, 5120)])
def test_big_shape_matvec(t, rows, cols):
    raw, x, want, scale = _big_matvec_case(t, rows, cols, seed=rows ^ cols)
    h = C.c_void_p()
    buf = np.frombuffer(raw, dtype=np.uint8)
    runtime.check(runtime.lib().evl_qmatrix_create(t, rows, cols, C.c_void_p(buf.ctypes.data), 0, C.byref(h)))
    try:
        dx, dy = gu.to_dev(x), gu.empty_f32(rows)
        for _ in range(2):  # the second launch reuses the first one's buffers
            runtime.check(runtime.lib().evl_qmatrix_matvec(h, gu.ptr(dx), gu.ptr(dy), None))
            gu.sync()
            got = dy.cpu().numpy().astype(np.float64)
            assert np.all(np.abs(got - want) <= 5e-5 * scale + 1e-7), float(np.abs(got - want).max())
    finally:
        runtime.lib().evl_qmatrix_free(h)
