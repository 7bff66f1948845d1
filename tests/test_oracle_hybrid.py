"""The oracle's Qwen3.5 hybrid path (src/runtime.rs:455-630, 684-695, 753-761), pinned:

1. the reference's own unit tests of the path (src/runtime.rs:843-860: the gated delta
   rule updates the state before the query read-out; interleaved rotary positions leave
   the non-rotary dimensions alone), restated against the oracle;
2. a float64 numpy restatement of a whole hybrid step -- gated-delta layers (causal
   depthwise conv, L2-normalised q/k, decay exp(softplus(alpha + dt) * a), the delta rule,
   per-head RMSNorm times SiLU(z)) and the gated full-attention layer with interleaved
   rotary positions -- written independently from the reference's description, over the
   oracle's own dequantised weights: logits within 1e-3 over 12 steps;
3. the loader's checks (runtime.rs:225-235, 278-290, 298-340) as error kinds.
"""
import numpy as np
import pytest

from evelyn_b200 import synth
from oracle import oracle as orc


def test_gated_delta_updates_state_before_query_readout():  # src/runtime.rs:843-851
    state = np.zeros(4, dtype=np.float32)
    out = orc.gated_delta_step(state, [1.0, 0.0], [1.0, 0.0], [2.0, -4.0], 1.0, 1.0)
    scale = 1.0 / np.sqrt(np.float32(2.0))
    assert abs(out[0] - 2.0 * scale) < 1e-6
    assert abs(out[1] + 4.0 * scale) < 1e-6
    assert state.tolist() == [2.0, -4.0, 0.0, 0.0]


def test_interleaved_rope_leaves_non_rotary_dimensions_untouched():  # src/runtime.rs:853-860
    values = orc.rope_interleaved(np.array([1.0, 0.0, 3.0, 4.0], dtype=np.float32), 1, 4, 2, 1, 10000.0)
    assert abs(values[0] - np.cos(np.float32(1.0))) < 1e-6
    assert abs(values[1] - np.sin(np.float32(1.0))) < 1e-6
    assert values[2:].tolist() == [3.0, 4.0]


# ------------------------------------------------------------ float64 restatement
def _sig(x):
    return 1.0 / (1.0 + np.exp(-x))


def _rms(x, w, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * w


class _Ref:
    """A hybrid Qwen3.5 decoder in float64 over the oracle's dequantised weights."""

    def __init__(self, m: orc.Model, spec: synth.ModelSpec):
        self.m, self.s = m, spec
        self.t = lambda n: m.tensor_f32(n).astype(np.float64)
        self.kv = [[] for _ in range(spec.layers)]
        kw, vw = spec.ssm_state * spec.ssm_groups, spec.ssm_inner
        self.channels = 2 * kw + vw
        self.hist = [np.zeros((spec.ssm_conv_kernel - 1, self.channels)) for _ in range(spec.layers)]
        vd = vw // spec.ssm_value_heads
        self.state = [np.zeros((spec.ssm_value_heads, spec.ssm_state, vd)) for _ in range(spec.layers)]
        self.pos = 0

    def W(self, name, rows):
        return self.t(name).reshape(rows, -1)

    def delta(self, li, xn):
        s, p = self.s, f"blk.{li}."
        kd, kh, vh = s.ssm_state, s.ssm_groups, s.ssm_value_heads
        vd, kw = s.ssm_inner // vh, s.ssm_state * s.ssm_groups
        proj = self.W(p + "attn_qkv.weight", self.channels) @ xn
        z = self.W(p + "attn_gate.weight", s.ssm_inner) @ xn
        conv = self.t(p + "ssm_conv1d.weight").reshape(self.channels, s.ssm_conv_kernel)
        inp = np.vstack([self.hist[li], proj[None, :]])  # [kernel][channels], oldest first
        c = (inp.T * conv).sum(axis=1)
        c = c * _sig(c)
        self.hist[li] = inp[1:]
        alpha = self.W(p + "ssm_alpha.weight", vh) @ xn
        beta = self.W(p + "ssm_beta.weight", vh) @ xn
        a, dt = self.t(p + "ssm_a"), self.t(p + "ssm_dt")
        out = np.zeros(s.ssm_inner)
        for h in range(vh):
            g = h % kh
            q = c[g * kd:(g + 1) * kd]
            k = c[kw + g * kd:kw + (g + 1) * kd]
            v = c[2 * kw + h * vd:2 * kw + (h + 1) * vd]
            q = q / np.sqrt(q @ q + s.eps)
            k = k / np.sqrt(k @ k + s.eps)
            decay = np.exp(np.log1p(np.exp(alpha[h] + dt[h])) * a[h])
            S = self.state[li][h] * decay
            S += np.outer(k, (v - k @ S) * _sig(beta[h]))
            self.state[li][h] = S
            out[h * vd:(h + 1) * vd] = (q @ S) / np.sqrt(kd)
        norm = self.t(p + "ssm_norm.weight")
        for h in range(vh):
            o = out[h * vd:(h + 1) * vd]
            zz = z[h * vd:(h + 1) * vd]
            out[h * vd:(h + 1) * vd] = _rms(o, norm, s.eps) * zz * _sig(zz)
        return self.W(p + "ssm_out.weight", s.dim) @ out

    def rope(self, v, heads):
        hd = self.s.head_dim
        rd = min(self.s.rope_dim or hd, hd) & ~1
        v = v.reshape(heads, hd).copy()
        for i in range(0, rd, 2):
            th = self.pos * self.s.rope_base ** (-i / rd)
            a, b = v[:, i].copy(), v[:, i + 1].copy()
            v[:, i], v[:, i + 1] = a * np.cos(th) - b * np.sin(th), a * np.sin(th) + b * np.cos(th)
        return v

    def full(self, li, xn):
        s, p = self.s, f"blk.{li}."
        H, KH, hd = s.heads, s.kv_heads, s.head_dim
        qg = (self.W(p + "attn_q.weight", 2 * H * hd) @ xn).reshape(H, 2, hd)
        q, gate = qg[:, 0], qg[:, 1]
        k = (self.W(p + "attn_k.weight", KH * hd) @ xn).reshape(KH, hd)
        v = (self.W(p + "attn_v.weight", KH * hd) @ xn).reshape(KH, hd)
        qn, kn = self.t(p + "attn_q_norm.weight"), self.t(p + "attn_k_norm.weight")
        q = np.stack([_rms(r, qn, s.eps) for r in q])
        k = np.stack([_rms(r, kn, s.eps) for r in k])
        q, k = self.rope(q.ravel(), H), self.rope(k.ravel(), KH)
        self.kv[li].append((k, v))
        K = np.stack([e[0] for e in self.kv[li]])
        V = np.stack([e[1] for e in self.kv[li]])
        att = np.zeros((H, hd))
        for h in range(H):
            kvh = h // (H // KH)
            sc = K[:, kvh] @ q[h] / np.sqrt(hd)
            w = np.exp(sc - sc.max())
            att[h] = (w / w.sum()) @ V[:, kvh] * _sig(gate[h])
        return self.W(p + "attn_output.weight", s.dim) @ att.ravel()

    def step(self, tok):
        s = self.s
        x = self.W("token_embd.weight", s.vocab)[tok].copy()
        for li in range(s.layers):
            p = f"blk.{li}."
            xn = _rms(x, self.t(p + "attn_norm.weight"), s.eps)
            delta = (li + 1) % s.full_attention_interval != 0
            x = x + (self.delta(li, xn) if delta else self.full(li, xn))
            fin = _rms(x, self.t(p + "post_attention_norm.weight"), s.eps)
            g = self.W(p + "ffn_gate.weight", s.ffn) @ fin
            u = self.W(p + "ffn_up.weight", s.ffn) @ fin
            x = x + self.W(p + "ffn_down.weight", s.dim) @ (g / (1 + np.exp(-g)) * u)
        self.pos += 1
        return self.W("output.weight", s.vocab) @ _rms(x, self.t("output_norm.weight"), s.eps)


ODD = dict(ssm_conv_kernel=2, ssm_groups=1, ssm_value_heads=3, ssm_inner=192, full_attention_interval=2)


@pytest.mark.parametrize("interleaved,rope_dim,kw", [(True, 0, {}), (False, 32, {}), (True, 0, ODD),
                                                     (True, 0, dict(full_attention_interval=1)),
                                                     (True, 64, dict(head_dim=256))])
def test_hybrid_step_matches_float64_restatement(interleaved, rope_dim, kw):
    spec = synth.qwen35_tiny(seed=21, mrope_interleaved=interleaved, rope_dim=rope_dim, **kw)
    m = orc.Model(synth.build(spec))
    assert m.cfg.full_attention_interval == spec.full_attention_interval
    assert m.cfg.ssm_value_heads == spec.ssm_value_heads
    ref, sess = _Ref(m, spec), orc.Session(m)
    if not interleaved:  # the NeoX split-half rotation
        def rope(v, heads):
            hd, rd = spec.head_dim, rope_dim
            v = v.reshape(heads, hd).copy()
            half = rd // 2
            for i in range(half):
                th = ref.pos * spec.rope_base ** (-2 * i / rd)
                a, b = v[:, i].copy(), v[:, i + half].copy()
                v[:, i], v[:, i + half] = a * np.cos(th) - b * np.sin(th), a * np.sin(th) + b * np.cos(th)
            return v
        ref.rope = rope
    worst = 0.0
    for tok in np.random.default_rng(3).integers(0, spec.vocab, 12):
        got, want = sess.step(int(tok)), ref.step(int(tok))
        worst = max(worst, float(np.abs(got - want).max()))
    assert worst < 1e-3, worst


def _patch(img_bytes: bytes, old: bytes, new: bytes) -> bytes:
    assert img_bytes.count(old) == 1 and len(old) == len(new)
    return img_bytes.replace(old, new)


def test_hybrid_loader_checks():
    spec = synth.qwen35_tiny(seed=2)
    img = synth.build(spec)  # the image owns the memory the array views
    raw = img.array().tobytes()
    # interval key 4 -> 2: layer 1 (index 1) should then be full attention
    key = b"qwen35.full_attention_interval"
    i = raw.index(key) + len(key)
    bad = raw[:i + 4] + (2).to_bytes(4, "little") + raw[i + 8:]
    with pytest.raises(orc.OracleError) as e:
        orc.Model(bad)
    assert e.value.kind == "InvalidData" and "full_attention_interval=2" in str(e.value)
    # SSM metadata missing
    with pytest.raises(orc.OracleError) as e:
        orc.Model(_patch(raw, b"qwen35.ssm.conv_kernel", b"qwen35.ssm.conv_kernex"))
    assert e.value.kind == "InvalidData" and "ssm.conv_kernel" in str(e.value)
    # value heads that do not divide the inner size
    key = b"qwen35.ssm.time_step_rank"
    i = raw.index(key) + len(key)
    bad = raw[:i + 4] + (3).to_bytes(4, "little") + raw[i + 8:]
    with pytest.raises(orc.OracleError) as e:
        orc.Model(bad)
    assert e.value.kind == "InvalidData"


def test_hybrid_session_state_is_per_session():
    spec = synth.qwen35_tiny(seed=5)
    m = orc.Model(synth.build(spec))
    a, b = orc.Session(m), orc.Session(m)
    for t in [1, 2, 3]:
        a.step(t)
    fresh = orc.Session(m)
    assert np.array_equal(b.step(7), fresh.step(7))
