/*
 * oracle.h -- C interface of the CPU oracle for Evelyn's decode token loop.
 *
 * TEST INFRASTRUCTURE ONLY. This library restates, in plain C++ on the CPU,
 * the reference's GGUF reader/dequantisers (src/gguf.rs) and its transformer
 * runtime (src/runtime.rs). It exists to check the CUDA engine and to time
 * the reference algorithm on host cores. Nothing in the product links it.
 *
 * Status codes mirror the io::ErrorKind values the reference returns:
 *   0 ok, 1 InvalidInput, 2 InvalidData, 3 NotFound, 4 Unsupported, 5 Io.
 */
#ifndef EVELYN_ORACLE_H
#define EVELYN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_model orc_model;
typedef struct orc_session orc_session;

/* FFN hook: mirrors `FfnBackend::ffn(layer, x) -> Vec<f32>` (runtime.rs:138).
 * Return 0 to use y; non-zero means "no answer" and the oracle runs the
 * dense FFN instead (the fallback RemoteAarnnFfn takes, remote.rs:247-271). */
typedef int (*orc_ffn_fn)(void* ctx, size_t layer, const float* x, size_t n, float* y);

typedef struct {
    char arch[64];
    uint64_t layers, dim, ffn, heads, kv_heads, head_dim, rope_dim, vocab;
    float rope_base, eps;
    int32_t rope_interleaved;
    int64_t eos_token_id; /* -1 when absent */
    uint64_t full_attention_interval;
    uint64_t ssm_conv_kernel, ssm_inner, ssm_state, ssm_groups, ssm_value_heads; /* 0 without SSM metadata */
} orc_config;

const char* orc_last_error(void);
void orc_set_threads(int n);
int orc_get_threads(void);

/* gguf.rs:288 type_bytes; returns -1 for unsupported types */
int64_t orc_type_bytes(uint32_t ggml_type, uint64_t n);
/* gguf.rs:300 f16_to_f32 */
float orc_f16_to_f32(uint16_t h);
/* gguf.rs:338 dequantize: raw has nbytes bytes, n values are expected. */
int orc_dequantize(uint32_t ggml_type, const uint8_t* raw, size_t nbytes, size_t n, float* out);

/* runtime.rs:199 Model::load, from a path or from a GGUF image in memory
 * (the memory must outlive the model). */
int orc_model_load(const char* path, orc_model** out);
int orc_model_load_memory(const uint8_t* data, size_t len, orc_model** out);
void orc_model_free(orc_model* m);
int orc_model_config(const orc_model* m, orc_config* out);
/* runtime.rs:409 Model::dense_ffn and :422 Model::ffn_input */
int orc_dense_ffn(const orc_model* m, size_t layer, const float* x, float* y);
int orc_ffn_input(const orc_model* m, size_t layer, const float* x, float* y);
/* QMatrix::matvec (runtime.rs:72) of a named 2-D tensor */
int orc_matvec(const orc_model* m, const char* tensor, const float* x, size_t xn, float* y, size_t yn);
/* dequantise a whole named tensor (gguf.rs:199 tensor_f32) */
int orc_tensor_f32(const orc_model* m, const char* tensor, float* out, size_t n);
int orc_tensor_info(const orc_model* m, const char* tensor, uint32_t* type, uint64_t* dims, uint32_t* ndims);

/* runtime.rs:643 Session::new, :773 Session::step */
int orc_session_new(const orc_model* m, orc_session** out);
void orc_session_free(orc_session* s);
uint64_t orc_session_pos(const orc_session* s);
int orc_session_step(orc_session* s, uint32_t token, orc_ffn_fn ffn, void* ctx, float* logits);
/* Timing aid for the CPU baseline: append `n` positions of seeded synthetic
 * K/V rows to every layer's cache, so a step can be timed at a given context
 * without running the prefix through the model. */
int orc_session_fill_kv(orc_session* s, uint64_t n, uint64_t seed);

/* runtime.rs:125, :897, :908 */
int orc_validate_token_ids(const uint32_t* ids, size_t n, size_t vocab);
/* runtime.rs:493-528 and 455-474, for their known-answer tests */
void orc_gated_delta_step(float* state, const float* q, const float* k, const float* v, size_t width, size_t nv,
                          float decay, float beta, float* out);
void orc_rope_interleaved(float* v, size_t heads, size_t hd, size_t rotary_dim, size_t pos, float base);
uint32_t orc_argmax(const float* v, size_t n);
uint32_t orc_sample_token(const float* logits, size_t n, float temperature, uint64_t* state);
float orc_log_prob(const float* logits, size_t n, uint32_t target);

#ifdef __cplusplus
}
#endif
#endif
