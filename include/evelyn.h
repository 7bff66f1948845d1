/*
 * evelyn.h -- C ABI of the B200 decode engine for Evelyn's token loop.
 *
 * Every entry point is a drop-in for one item of the reference's Rust runtime
 * API (paths below are inside the neuralmimicry/evelyn tree). A Rust FFI crate
 * binds these one-to-one.
 *
 * Conventions
 *   - Plain pointers and sizes only. "host" buffers are ordinary CPU memory;
 *     "device" buffers are CUDA device pointers on the model's device.
 *   - Every call returns an evl_status. On failure evl_last_error() holds a
 *     message (thread-local). Status codes map one-to-one to the io::ErrorKind
 *     values the reference returns (src/gguf.rs, src/runtime.rs).
 *   - No CPU fallback exists: without a usable CUDA device every call that
 *     needs one fails with EVL_ERR_CUDA.
 */
#ifndef EVELYN_H
#define EVELYN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EVL_ABI_VERSION 1

typedef enum evl_status {
    EVL_OK = 0,
    EVL_ERR_INVALID_INPUT = 1, /* io::ErrorKind::InvalidInput (runtime.rs:125-135, :55-63) */
    EVL_ERR_INVALID_DATA = 2,  /* io::ErrorKind::InvalidData  (bad GGUF, shapes, metadata) */
    EVL_ERR_NOT_FOUND = 3,     /* io::ErrorKind::NotFound     (gguf.rs:203-205) */
    EVL_ERR_UNSUPPORTED = 4,   /* io::ErrorKind::Unsupported  (gguf.rs:280-285) */
    EVL_ERR_IO = 5,            /* any other io::Error (file access, short reads) */
    EVL_ERR_CUDA = 6,          /* CUDA runtime / device error (no CPU counterpart) */
    EVL_ERR_OUT_OF_MEMORY = 7, /* device or pinned-host allocation failed */
    EVL_ERR_NCCL = 8,          /* tensor-parallel collective failed */
    EVL_ERR_TIMEOUT = 9        /* a bounded device wait gave up */
} evl_status;

typedef struct evl_model evl_model;
typedef struct evl_session evl_session;
typedef struct evl_batch evl_batch;
typedef struct evl_qmatrix evl_qmatrix;
typedef struct evl_remote_ffn evl_remote_ffn;

/* Mirrors `pub struct Config` (src/runtime.rs:93-110) for the dense-attention path. */
typedef struct evl_config {
    char arch[64];
    uint64_t layers, dim, ffn, heads, kv_heads, head_dim, rope_dim, vocab;
    float rope_base, eps;
    int32_t rope_interleaved;
    int64_t eos_token_id; /* -1 when the GGUF has none */
} evl_config;

typedef struct evl_model_options {
    uint32_t struct_size; /* sizeof(evl_model_options) */
    int32_t device;       /* CUDA device ordinal; -1 = the calling thread's current device */
    int32_t tp_rank;      /* tensor-parallel rank in [0, tp_size) */
    int32_t tp_size;      /* 1 = one GPU; 2/4/8 = Megatron split over that many ranks */
    uint8_t nccl_id[128]; /* evl_tp_unique_id() of rank 0, shared with every rank (tp_size > 1) */
    uint32_t kv_f32;      /* 1: keep the KV cache in f32 like the reference; 0: f16 pages */
    uint32_t reserved[7];
} evl_model_options;

/* FfnBackend (src/runtime.rs:138-140). `ffn` receives the normalised FFN input x of
 * width n (what Model::ffn_input returns, runtime.rs:422) in host memory and writes
 * the FFN output y (width n). Return values:
 *   0             y holds the answer (RemoteAarnnFfn success, remote.rs:253);
 *   EVL_FFN_DENSE run the model's dense FFN for this layer on the device (DenseFfn,
 *                 CaptureFfn: runtime.rs:428-434, remote.rs:35-45);
 *   anything else failure: the engine runs the dense FFN and increments
 *                 *fallbacks (the fallback of remote.rs:254-268).
 * `routed[layer] != 0` selects the layers that call `ffn`; the others stay dense on
 * the device with no host round trip. routed == NULL routes every layer. */
#define EVL_FFN_DENSE 1
typedef int (*evl_ffn_fn)(void* ctx, size_t layer, const float* x, size_t n, float* y);
typedef struct evl_ffn_backend {
    evl_ffn_fn ffn;
    void* ctx;
    const uint8_t* routed;
    size_t routed_len;
    uint64_t* fallbacks; /* optional */
} evl_ffn_backend;

/* ------------------------------------------------------------------ library */
const char* evl_last_error(void);
uint32_t evl_abi_version(void);
void evl_model_options_init(evl_model_options* opts);
/* validate_token_ids (src/runtime.rs:125-135) */
evl_status evl_validate_token_ids(const uint32_t* ids, size_t n, size_t vocab);
/* argmax (src/runtime.rs:897-905): first maximum, strict '>' from f32::MIN. host */
uint32_t evl_argmax(const float* logits, size_t n);
/* log_prob (src/runtime.rs:908-912). host */
float evl_log_prob(const float* logits, size_t n, uint32_t target);
/* ncclGetUniqueId for tensor parallelism: rank 0 calls it and shares the bytes. */
evl_status evl_tp_unique_id(uint8_t out[128]);
/* The tensor-parallel shard that rank `rank` of `tp_size` loads (the Megatron split that
 * stands in for one process running src/runtime.rs:773-808): [first, last) rows of
 * attn_q (and input columns of attn_output), of attn_k / attn_v, of ffn_gate / ffn_up
 * (and input columns of ffn_down, on 256-value super-block boundaries, uneven when the
 * block count does not divide) and of the LM head. Host only; uses heads, kv_heads,
 * head_dim, ffn and vocab of cfg. InvalidInput / Unsupported as evl_model_load. */
typedef struct evl_tp_shard {
    uint64_t q_rows[2], kv_rows[2], ffn_rows[2], vocab_rows[2];
} evl_tp_shard;
evl_status evl_tp_shard_plan(const evl_config* cfg, int32_t tp_size, int32_t rank, evl_tp_shard* out);

/* ------------------------------------------------------------------ model */
/* Model::load (src/runtime.rs:199-406). Weights stay quantised, repacked in HBM. */
evl_status evl_model_load(const char* path, const evl_model_options* opts, evl_model** out);
/* Same, from a GGUF image already in host memory (not retained after return). */
evl_status evl_model_load_memory(const void* data, size_t len, const evl_model_options* opts, evl_model** out);
void evl_model_free(evl_model* model);
/* Model.cfg (src/runtime.rs:185) */
evl_status evl_model_config(const evl_model* model, evl_config* out);
/* Config::full_attention_interval and SsmConfig (src/runtime.rs:106-120) of a Qwen3.5
 * ("qwen35") model, whose layers are gated-delta layers except every interval-th one
 * (gated full attention). All zero but full_attention_interval for other models. */
typedef struct evl_ssm_config {
    int32_t has_ssm;
    uint32_t delta_layers; /* layers with Attention::GatedDelta */
    uint64_t full_attention_interval;
    uint64_t conv_kernel, inner, state, groups, value_heads;
} evl_ssm_config;
evl_status evl_model_ssm_config(const evl_model* model, evl_ssm_config* out);
/* Model::dense_ffn (src/runtime.rs:409-418): host x[dim] -> host y[dim], on the device.
 * With tp_size > 1 every rank must make the same call (it runs a collective). */
evl_status evl_model_dense_ffn(evl_model* model, size_t layer, const float* x, float* y);
/* Model::ffn_input (src/runtime.rs:422-424): rms_norm(x, ffn_norm). host -> host */
evl_status evl_model_ffn_input(evl_model* model, size_t layer, const float* x, float* y);
/* Gguf::tensor_f32 (src/gguf.rs:199-215) of a model tensor, dequantised exactly on the
 * device from the repacked weights. n must equal the element count (this rank's shard
 * under tensor parallelism). host out */
evl_status evl_model_dequantize(evl_model* model, const char* tensor, float* out, size_t n);
/* QMatrix::matvec (src/runtime.rs:72-88) of one model matrix. host x[cols] -> host y[rows] */
evl_status evl_model_matvec(evl_model* model, const char* tensor, const float* x, size_t xn, float* y, size_t yn);
/* Bytes of quantised weights one decode step streams from HBM on this rank. */
uint64_t evl_model_weight_bytes(const evl_model* model);

/* ------------------------------------------------------------------ session (one sequence) */
/* Session::new (src/runtime.rs:643-660); max_ctx bounds the paged KV cache. */
evl_status evl_session_new(evl_model* model, uint32_t max_ctx, evl_session** out);
void evl_session_free(evl_session* s);
/* Session.pos (src/runtime.rs:639) */
uint64_t evl_session_pos(const evl_session* s);
/* Session::step (src/runtime.rs:773-808). ffn == NULL is DenseFfn on every layer.
 * logits_out (host, vocab floats) and argmax_out (host) are each optional. */
evl_status evl_session_step(evl_session* s, uint32_t token, const evl_ffn_backend* ffn, float* logits_out,
                            uint32_t* argmax_out);
/* The greedy loop of src/bin/evelyn-generate.rs:81-86 without host round trips:
 * feeds `token`, then n-1 times the argmax of the previous step; tokens_out[i] is the
 * argmax after step i (n entries, host). Dense FFN on every layer. */
evl_status evl_session_generate(evl_session* s, uint32_t token, uint32_t n, uint32_t* tokens_out);
/* Prompt processing: feeds tokens[0 .. n) as n evl_session_step calls would (the loop
 * of src/bin/evelyn-generate.rs:69-80, one Session::step per prompt token), but in
 * batched steps of up to 32 prompt positions whose products run on the tensor cores.
 * logits_out ([n][vocab], host) and argmax_out ([n], host) are each optional: row i is
 * what step i would have returned. Dense FFN on every layer. Under tensor parallelism
 * every rank makes the same call. Models without the tensor-core products (Qwen3.5
 * hybrid layers, unquantised matrices) take the prompt one step per token. */
evl_status evl_session_prefill(evl_session* s, const uint32_t* tokens, size_t n, float* logits_out,
                               uint32_t* argmax_out);
/* sample_token (src/server.rs:326-352) on the device, from the logits of the session's
 * last step, so the logits never cross to the host: temperature <= FLT_EPSILON gives
 * the step's greedy pick and leaves *rng_state alone; otherwise *rng_state (the
 * xorshift64* state the caller keeps per request, host in/out) advances once and
 * *token_out (host) is the first index whose running sum of exp((v - max) / T)
 * reaches the draw times the total (the greedy pick if the total is not finite and
 * positive). Feeding the token and stopping at the model's eos_token_id
 * (server.rs:514-519) stay with the caller. */
evl_status evl_session_sample(evl_session* s, float temperature, uint64_t* rng_state, uint32_t* token_out);
/* Device CUDA stream the session launches on (cudaStream_t), for event timing. */
void* evl_session_stream(evl_session* s);
/* Number of engine kernels one dense step launches (known after the first step). */
uint32_t evl_session_kernels_per_step(const evl_session* s);
/* Human-readable notes on the launches the session's step uses (the opt-in persistent
 * step kernel) and, where one is not used, why; empty when there is nothing to say.
 * Valid until the next call on the session or its release. */
const char* evl_session_notes(const evl_session* s);

/* ------------------------------------------------------------------ batched decode */
/* n_seqs independent Sessions stepped together (one token each per step), sharing
 * every weight read. Dense FFN on every layer. */
evl_status evl_batch_new(evl_model* model, uint32_t n_seqs, uint32_t max_ctx, evl_batch** out);
void evl_batch_free(evl_batch* b);
uint64_t evl_batch_pos(const evl_batch* b, uint32_t seq);
/* tokens[n_seqs] (host) in; logits_out [n_seqs][vocab] and argmax_out [n_seqs], both optional (host). */
evl_status evl_batch_step(evl_batch* b, const uint32_t* tokens, float* logits_out, uint32_t* argmax_out);
void* evl_batch_stream(evl_batch* b);
/* evl_session_prefill for sequence `seq` of a batch: its prompt tokens[0 .. n) in batched
 * steps of up to 32 positions on the tensor cores; the other sequences are untouched.
 * logits_out ([n][vocab]) and argmax_out ([n]) are optional (host). EVL_ERR_UNSUPPORTED
 * for a batch of several sequences of a model without the tensor-core products. */
evl_status evl_batch_prefill(evl_batch* b, uint32_t seq, const uint32_t* tokens, size_t n, float* logits_out,
                             uint32_t* argmax_out);
/* evl_session_sample for every sequence of a batch: rng_states[n_seqs] (host in/out),
 * tokens_out[n_seqs] (host). */
evl_status evl_batch_sample(evl_batch* b, float temperature, uint64_t* rng_states, uint32_t* tokens_out);

/* ------------------------------------------------------------------ kernels on caller buffers */
/* dequantize (src/gguf.rs:338-430) of raw GGUF blocks: d_raw holds type_bytes(type, n)
 * bytes; d_out receives n floats. Bit-exact. device pointers; stream may be NULL. */
evl_status evl_dequantize_raw(uint32_t ggml_type, const void* d_raw, size_t n, float* d_out, void* stream);
/* A standalone quantised matrix (QMatrix, src/runtime.rs:23-51) built from host GGUF
 * bytes [rows][type_bytes(type, cols)] on `device`. */
evl_status evl_qmatrix_create(uint32_t ggml_type, uint32_t rows, uint32_t cols, const void* host_raw, int device,
                              evl_qmatrix** out);
void evl_qmatrix_free(evl_qmatrix* m);
uint64_t evl_qmatrix_bytes(const evl_qmatrix* m);
/* y = W x (QMatrix::matvec, runtime.rs:72-88). device pointers, x 16-byte aligned;
 * stream may be NULL. On a non-NULL stream the launch may begin (streaming weights)
 * while the stream's previous kernel finishes; it reads x and writes y only after that
 * kernel has completed. */
evl_status evl_qmatrix_matvec(const evl_qmatrix* m, const float* d_x, float* d_y, void* stream);
/* QMatrix::matvec (runtime.rs:72-88) of nvec (1..32) vectors at once, as a Batch step
 * needs: d_x [nvec][cols] -> d_y [nvec][rows], on the tensor cores (the first call
 * also builds the matrix's GEMM-layout copy). cols must be a multiple of 256; types
 * Q4_K, Q6_K, Q8_0. Synchronises `stream`. */
evl_status evl_qmatrix_matmul(evl_qmatrix* m, const float* d_x, uint32_t nvec, float* d_y, void* stream);
/* exact dequantisation of all rows to d_out [rows][cols]. device pointers */
evl_status evl_qmatrix_dequantize(const evl_qmatrix* m, float* d_out, void* stream);
/* GQA decode attention for one new position (the attention core of full_attention,
 * runtime.rs:723-766) over a paged KV cache of f16 rows:
 *   d_q        [heads][head_dim] f32, already normed and rotated
 *   d_k_pages  [n_pages][kv_heads][page_size][head_dim] f16, likewise d_v_pages
 *   d_page_table [ceil(t / page_size)] int32 page ids, t = positions to attend
 *   d_out      [heads][head_dim] f32
 * head_dim must be 64, 128 or 256 and page_size 16. Allocates its split scratch per call
 * and synchronises `stream` before returning. */
evl_status evl_attention_decode(const float* d_q, const void* d_k_pages, const void* d_v_pages,
                                const int32_t* d_page_table, uint32_t t, uint32_t heads, uint32_t kv_heads,
                                uint32_t head_dim, uint32_t page_size, float* d_out, void* stream);
/* Bytes of device workspace evl_attention_decode_ws needs for up to t_max positions. */
size_t evl_attention_workspace_bytes(uint32_t t_max, uint32_t heads, uint32_t kv_heads, uint32_t head_dim);
/* evl_attention_decode with the split scratch in a caller-allocated device workspace
 * (256-byte aligned, evl_attention_workspace_bytes(t_max, ...) bytes, t <= t_max);
 * asynchronous on `stream`. The workspace's first int32 is a device error flag the
 * kernel sets (2) if a wait for KV pages timed out; the caller clears it. */
evl_status evl_attention_decode_ws(const float* d_q, const void* d_k_pages, const void* d_v_pages,
                                   const int32_t* d_page_table, uint32_t t, uint32_t heads, uint32_t kv_heads,
                                   uint32_t head_dim, uint32_t page_size, float* d_out, void* d_workspace,
                                   size_t workspace_bytes, void* stream);
/* evl_attention_decode without any device allocation (no counterpart in the reference,
 * whose attention runs on the host). For callers that may not allocate device memory
 * during a decode call: a process whose HBM belongs to its own pool, or one that must
 * not let a cudaFree synchronise the device mid-step. The split scratch is a fixed
 * 1.5 MiB array per device inside this library; a shape needing more is rejected
 * with EVL_ERR_INVALID_INPUT (on a 148-SM B200 every accepted shape fits). The call
 * clears the scratch's error flag itself and synchronises `stream` before returning.
 * The first call on a device resolves the array's address (set-up). Every call reads
 * the error flag back to the host and synchronises `stream`, so it cannot be used
 * inside a stream capture (evl_attention_decode_ws is the asynchronous variant).
 * Calls on one device that overlap in time race on the shared scratch; the caller
 * serialises them. Same arguments and results as evl_attention_decode. */
evl_status evl_attention_decode_noalloc(const float* d_q, const void* d_k_pages, const void* d_v_pages,
                                        const int32_t* d_page_table, uint32_t t, uint32_t heads, uint32_t kv_heads,
                                        uint32_t head_dim, uint32_t page_size, float* d_out, void* stream);

/* ------------------------------------------------------------------ AARNN routing (src/remote.rs) */
typedef struct evl_endpoint_stats { /* EndpointStats, remote.rs:13-24 */
    uint64_t calls, failures, retries;
    uint64_t total_ns, max_ns;
} evl_endpoint_stats;
/* RemoteAarnnFfn::new (remote.rs:185-205): layers[i] is served by the AARNN region at
 * addrs[i] ("host:port") over the wire protocol of remote.rs:69-111, with one
 * reconnect and a dense fallback; timeout_ms is the read timeout. model may be NULL,
 * in which case the routed layers are not checked against a model's layer count. */
evl_status evl_remote_ffn_new(evl_model* model, size_t n, const size_t* layers, const char* const* addrs,
                              uint32_t timeout_ms, evl_remote_ffn** out);
void evl_remote_ffn_free(evl_remote_ffn* r);
/* The evl_ffn_backend that routes the configured layers through `r`. */
evl_status evl_remote_ffn_backend(evl_remote_ffn* r, evl_ffn_backend* out);
/* RemoteAarnnFfn.fallbacks (remote.rs:166) */
uint64_t evl_remote_ffn_fallbacks(const evl_remote_ffn* r);
/* endpoint_stats (remote.rs:236-244) for one routed layer */
evl_status evl_remote_ffn_stats(const evl_remote_ffn* r, size_t layer, evl_endpoint_stats* out);

#ifdef __cplusplus
}
#endif
#endif /* EVELYN_H */
