/*
 * synth_gguf.h -- seeded synthetic GGUF images for Qwen3 / Qwen3.5-family decoders, and
 * the GGUF block encoders behind them (the reference ships dequantisers only).
 * Tooling for tests and benchmarks; not part of the decode path.
 */
#ifndef EVELYN_SYNTH_GGUF_H
#define EVELYN_SYNTH_GGUF_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    char arch[32];            /* "qwen3" */
    uint32_t layers, dim, ffn, heads, kv_heads, head_dim, vocab;
    float rope_base, eps, stddev;
    uint32_t type_attn_q, type_attn_k, type_attn_v, type_attn_output;
    uint32_t type_ffn_gate, type_ffn_up, type_ffn_down, type_embed, type_output;
    uint32_t qk_norm;         /* write attn_q_norm / attn_k_norm */
    uint32_t tied_output;     /* omit output.weight (LM head = token_embd) */
    uint32_t eos_token_id;
    uint64_t seed;
    int32_t threads;          /* <= 0: all hardware threads */
    /* arch "qwen35" (runtime.rs:225-235, 276-371): layer i is a gated-delta layer unless
       (i + 1) % full_attention_interval == 0; full-attention layers carry the gated query
       (attn_q rows = 2 * heads * head_dim); every layer's FFN norm is post_attention_norm. */
    uint32_t full_attention_interval;
    uint32_t ssm_conv_kernel, ssm_state, ssm_groups, ssm_value_heads, ssm_inner;
    uint32_t type_ssm;        /* attn_qkv, attn_gate, ssm_alpha, ssm_beta, ssm_out */
    uint32_t rope_dim;        /* rope.dimension_count (0: not written, = head_dim) */
    uint32_t mrope_interleaved; /* rope.mrope_interleaved = true */
} evs_model_spec;

const char* evs_last_error(void);
/* Encode n f32 values as ggml `type` (Q8_0, Q4_K, Q5_K, Q6_K, F16, BF16, F32). */
int evs_encode(uint32_t type, const float* x, size_t n, uint8_t* out, size_t out_len);
uint16_t evs_f32_to_f16(float f);
/* Build a complete GGUF v3 image in malloc'd memory; free with evs_free. */
int evs_build(const evs_model_spec* spec, uint8_t** out, size_t* out_len);
void evs_free(uint8_t* p);
int evs_write_file(const uint8_t* data, size_t len, const char* path);

#ifdef __cplusplus
}
#endif
#endif
