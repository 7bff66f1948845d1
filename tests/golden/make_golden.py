"""Regenerate the golden fixtures in this directory (run from the repository root):

    python tests/golden/make_golden.py

dequant_random.npz
    Random raw GGUF blocks (Q8_0, Q4_K, Q5_K, Q6_K; arbitrary quant bytes, finite f16
    scales including subnormals and -0) and their dequantised values from gguf-py's
    ``quants.dequantize`` (gguf 0.19.0), an implementation independent of the oracle.
tiny_qwen3_hf.npz
    Logits of the seeded tiny synthetic Qwen3 model (evelyn_b200.synth.tiny(seed=0))
    for a fixed token sequence, computed by HuggingFace transformers' Qwen3ForCausalLM
    in float32 with the dequantised GGUF weights -- an independent implementation of
    the architecture the reference's runtime.rs decodes (NeoX RoPE, QK-norm, GQA,
    SwiGLU, RMSNorm). Stores the GGUF image's sha256 so drift in the synthetic model
    is caught.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def random_blocks(ggml_type: int, nblocks: int, rng) -> np.ndarray:
    bb = {8: 34, 12: 144, 13: 176, 14: 210}[ggml_type]
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)

    def f16(v):
        return np.asarray(v, dtype=np.float16).view(np.uint8).reshape(-1, 2)

    if ggml_type == 8:
        raw[:, 0:2] = f16(rng.uniform(-0.05, 0.05, nblocks))
        off = 0
    elif ggml_type in (12, 13):
        raw[:, 0:2] = f16(rng.uniform(0, 0.01, nblocks))
        raw[:, 2:4] = f16(rng.uniform(0, 0.01, nblocks))
        off = 0
    else:
        raw[:, 208:210] = f16(rng.uniform(-0.01, 0.01, nblocks))
        off = 208
    raw[0, off:off + 2] = [0x01, 0x00]  # smallest subnormal
    raw[1, off:off + 2] = [0xff, 0x03]  # largest subnormal
    raw[2, off:off + 2] = [0x00, 0x80]  # -0
    return raw


def make_dequant():
    import gguf
    from gguf import quants
    rng = np.random.default_rng(2024)
    out = {}
    for t in (8, 12, 13, 14):
        raw = random_blocks(t, 64, rng)
        y = quants.dequantize(raw.reshape(-1), gguf.GGMLQuantizationType(t)).astype(np.float32).reshape(-1)
        out[f"raw_{t}"] = raw.reshape(-1)
        out[f"y_{t}"] = y
    np.savez_compressed(os.path.join(HERE, "dequant_random.npz"), **out)


def make_hf():
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from evelyn_b200 import synth
    from oracle import oracle as orc

    spec = synth.tiny(seed=0)
    img = synth.build(spec)
    digest = hashlib.sha256(img.array().tobytes()).hexdigest()
    m = orc.Model(img)
    c = m.cfg
    cfg = Qwen3Config(vocab_size=c.vocab, hidden_size=c.dim, intermediate_size=c.ffn, num_hidden_layers=c.layers,
                      num_attention_heads=c.heads, num_key_value_heads=c.kv_heads, head_dim=c.head_dim,
                      rms_norm_eps=c.eps, rope_theta=c.rope_base, tie_word_embeddings=False,
                      max_position_embeddings=4096, attention_bias=False)
    cfg._attn_implementation = "eager"
    hf = Qwen3ForCausalLM(cfg).float().eval()

    def W(name, rows, cols):
        return torch.from_numpy(m.tensor_f32(name).reshape(rows, cols).copy())

    def V(name):
        return torch.from_numpy(m.tensor_f32(name))

    qw, kw = c.heads * c.head_dim, c.kv_heads * c.head_dim
    sd = {"model.embed_tokens.weight": W("token_embd.weight", c.vocab, c.dim),
          "model.norm.weight": V("output_norm.weight"), "lm_head.weight": W("output.weight", c.vocab, c.dim)}
    for i in range(c.layers):
        p, h = f"blk.{i}.", f"model.layers.{i}."
        sd[h + "self_attn.q_proj.weight"] = W(p + "attn_q.weight", qw, c.dim)
        sd[h + "self_attn.k_proj.weight"] = W(p + "attn_k.weight", kw, c.dim)
        sd[h + "self_attn.v_proj.weight"] = W(p + "attn_v.weight", kw, c.dim)
        sd[h + "self_attn.o_proj.weight"] = W(p + "attn_output.weight", c.dim, qw)
        sd[h + "self_attn.q_norm.weight"] = V(p + "attn_q_norm.weight")
        sd[h + "self_attn.k_norm.weight"] = V(p + "attn_k_norm.weight")
        sd[h + "input_layernorm.weight"] = V(p + "attn_norm.weight")
        sd[h + "post_attention_layernorm.weight"] = V(p + "ffn_norm.weight")
        sd[h + "mlp.gate_proj.weight"] = W(p + "ffn_gate.weight", c.ffn, c.dim)
        sd[h + "mlp.up_proj.weight"] = W(p + "ffn_up.weight", c.ffn, c.dim)
        sd[h + "mlp.down_proj.weight"] = W(p + "ffn_down.weight", c.dim, c.ffn)
    hf.load_state_dict(sd, strict=True)
    tokens = np.random.default_rng(1).integers(0, c.vocab, 40).astype(np.int64)
    with torch.no_grad():
        logits = hf(torch.from_numpy(tokens)[None]).logits[0].numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "tiny_qwen3_hf.npz"), tokens=tokens, logits=logits,
                        gguf_sha256=np.array(digest))


if __name__ == "__main__":
    make_dequant()
    make_hf()
    print("fixtures written to", HERE)
