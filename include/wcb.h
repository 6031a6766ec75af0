/*
 * wcb.h — C ABI of the B200 (sm_100a) transformer token loop.
 *
 * Drop-in boundary for wasm-chord's `wasm-chord-runtime` Model / generate /
 * GenerationConfig path (crates/wasm-chord-runtime/src/transformer/model.rs).
 * Conventions copied from the reference C ABI:
 *   - every call returns a uint32 error code (ErrorCode, wasm-chord-runtime/src/lib.rs:80-89);
 *   - the message of the last failure on the calling thread is read with
 *     wcb_last_error (wasmchord_last_error, abi.rs:209-222);
 *   - model handles are uint32 > 0, 0 is never a valid handle (abi.rs:57-92).
 * All buffers in these signatures are HOST memory owned by the caller, except
 * where a parameter is documented as a device pointer. The library owns the
 * device weights, KV cache and CUDA graphs of each handle; wcb_model_free
 * releases them. One handle is one model replica on one GPU and is not
 * re-entrant (the reference's `&mut self`); distinct handles may be driven from
 * distinct threads.
 */
#ifndef WCB_H
#define WCB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ErrorCode — wasm-chord-runtime/src/lib.rs:80-89 */
enum {
  WCB_OK = 0,
  WCB_ERR_GENERIC = 1,
  WCB_ERR_OOM = 2,
  WCB_ERR_INVALID_ARGUMENT = 3,
  WCB_ERR_MODEL_PARSE = 4,
  WCB_ERR_BACKEND_UNSUPPORTED = 5,
  WCB_ERR_SHADER_COMPILE = 6, /* unused; kept so codes line up with the reference */
  WCB_ERR_IO = 7
};

/* GGUF tensor types of 2-D weights (gguf.rs:446-467; the raw blocks are
 * uploaded unchanged). wcb_gemv_dev takes the two quantised types only. */
enum { WCB_DTYPE_F32 = 0, WCB_DTYPE_F16 = 1, WCB_DTYPE_Q4_K = 12, WCB_DTYPE_Q6_K = 14 };

/* KV cache element type */
enum { WCB_KV_F32 = 0, WCB_KV_F16 = 1 };

/* Load options (no counterpart in the reference, whose Model::new takes only a
 * TransformerConfig: model.rs:188). Fill them with wcb_load_opts_init, which
 * writes the defaults and struct_size = sizeof(wcb_load_opts), then change the
 * fields you need. The library reads only the first struct_size bytes, so a
 * caller compiled against an older, shorter version of this struct keeps
 * working when fields are appended; fields beyond struct_size take their
 * defaults. struct_size must be at least WCB_LOAD_OPTS_V1_SIZE (the fields up to
 * and including tp_id). A NULL options pointer means all defaults. Layout: every
 * field is 4-byte aligned, no padding (see wcb_struct_layout). */
typedef struct wcb_load_opts {
  uint32_t struct_size; /* bytes of this struct the caller initialised */
  int32_t device;     /* CUDA device ordinal */
  uint32_t max_seq;   /* KV capacity in tokens; 0 = GGUF context_length (kv_cache.rs:48-53) */
  uint32_t kv_dtype;  /* WCB_KV_F32 (reference numerics) or WCB_KV_F16 */
  uint32_t max_batch; /* sequences per wcb_generate_batch call; 0 = 1 */
  uint32_t flags;     /* bit 0: no CUDA graphs for decode steps; bit 1: no programmatic
                         dependent launch; bit 2: no tensor-core GEMM for prefill (GEMV only);
                         bit 3: no persistent decode-step kernel (one launch per op instead);
                         bit 4: stream the layer weights from pinned host memory through a
                         two-layer device ring, one layer ahead of the compute (models that do
                         not fit in GPU memory; replaces the reference's Memory64 layer
                         manager, memory64_layer_manager.rs:76-300, async_prefetch.rs:83-190).
                         Single GPU, per-op kernels, no batched path;
                         bit 5: sampled decoding (temperature > 0) samples on the host from
                         each step's logits instead of on the device; both draw the same
                         tokens for a seed. */
  /* Tensor parallelism (one process per GPU; no counterpart in the reference, whose
     sharding.rs is bookkeeping only). tp_size 0 or 1: the whole model on `device`.
     tp_size > 1: this process holds rank tp_rank's shard (query/KV heads, o and down
     input columns, gate/up rows, LM-head vocabulary rows) and joins the NCCL group
     named by tp_id (from wcb_tp_id on one rank, shared by the caller); all ranks
     must make the same calls in the same order. */
  uint32_t tp_rank;
  uint32_t tp_size;
  uint8_t tp_id[128];
  /* Bound, in milliseconds, of every device-side wait on another rank's or
     another CTA's data (tensor-parallel partial sums, the decode step's tagged
     activations). A wait that runs out makes the call fail with
     WCB_ERR_BACKEND_UNSUPPORTED instead of hanging. 0 = 2000 ms; at most 60000. */
  uint32_t wait_ms;
} wcb_load_opts;

/* Bytes of the fields every caller must initialise (struct_size .. tp_id). */
#define WCB_LOAD_OPTS_V1_SIZE 160u

/* Defaults: device 0, max_seq = context_length, f32 KV cache, max_batch 1,
 * flags 0, one rank, wait_ms 2000; struct_size = sizeof(wcb_load_opts). */
void wcb_load_opts_init(wcb_load_opts* opts);

/* Size (field == NULL) or byte offset of a field of a struct of this header:
 * "wcb_load_opts", "wcb_gen_config" or "wcb_model_config". SIZE_MAX for an
 * unknown struct or field. A binding generated by hand (ctypes, Rust repr(C))
 * checks its own layout against these once at start-up. */
size_t wcb_struct_layout(const char* struct_name, const char* field);

/* TransformerConfig — transformer/config.rs:6-41 (plus head_dim) */
typedef struct wcb_model_config {
  uint32_t vocab_size, hidden_size, num_layers, num_heads, num_kv_heads;
  uint32_t intermediate_size, max_seq_len, head_dim;
  float rms_norm_eps, rope_theta;
} wcb_model_config;

/* GenerationConfig — transformer/config.rs:60-78, plus the sampler seed that
 * generate() hard-codes to 42 (model.rs:1336) and the EOS id that generate()
 * reads from the tokenizer (model.rs:1400). eos_id = UINT32_MAX disables EOS. */
typedef struct wcb_gen_config {
  uint32_t max_tokens;
  float temperature;
  float top_p;
  uint32_t top_k;
  float repetition_penalty;
  uint64_t seed;
  uint32_t eos_id;
} wcb_gen_config;

/* Fills the reference defaults: max_tokens 100, temperature 0.7, top_p 0.9,
 * top_k 40, repetition_penalty 1.1 (config.rs:74-78), seed 42, eos_id 2. */
void wcb_gen_config_default(wcb_gen_config* cfg);

/* Model::new + Model::load_from_gguf (model.rs:188, :364) from a GGUF file:
 * parses the header and config (gguf.rs:111-276), uploads raw Q4_K / Q6_K
 * blocks (Q6_K padded from 210 to 224 bytes for 16-byte alignment) and F32 /
 * F16 weights to HBM unchanged, allocates the device KV cache. Without an
 * output.weight the LM head is the reference's weight tying,
 * transpose_matrix(token embeddings, hidden, vocab) (model.rs:596-606). Models
 * with F32 / F16 2-D weights run the per-op kernels (no persistent decode step,
 * no batched decode step). Shapes the kernels cover: head_dim 64 or 128, hidden
 * and intermediate sizes multiples of 256, a vocabulary that is a multiple of 4,
 * at most 16 query heads per KV head; others are refused from the header with
 * WCB_ERR_BACKEND_UNSUPPORTED before any GPU call (inconsistent head counts:
 * WCB_ERR_INVALID_ARGUMENT). */
uint32_t wcb_model_load(const char* gguf_path, const wcb_load_opts* opts, uint32_t* out_handle);

/* Releases a handle (wasmchord_free_model, abi.rs:95-108). */
uint32_t wcb_model_free(uint32_t handle);

/* TransformerConfig of a loaded model. */
uint32_t wcb_model_config_get(uint32_t handle, wcb_model_config* out);

/* Model::forward (model.rs:832-1192): runs n tokens at `position`, appends their
 * K/V at the current KV length, writes the vocab_size logits of the LAST token
 * to logits_out (host). Errors: n == 0, or KV overflow (kv_cache.rs:48-53,
 * WCB_ERR_MODEL_PARSE as in the reference). */
uint32_t wcb_forward(uint32_t handle, const uint32_t* ids, size_t n, size_t position, float* logits_out);

/* Model::clear_kv_cache (model.rs:1547) and the KV length (KVCache::current_seq_len). */
uint32_t wcb_clear_kv(uint32_t handle);
uint32_t wcb_kv_len(uint32_t handle, size_t* out_len);

/* Model::generate (model.rs:1322-1415) on token ids: clears the KV cache,
 * prefills the prompt, samples the first token without an EOS check, then
 * decodes until cfg->max_tokens tokens or EOS (checked before the push).
 * Writes the generated ids (prompt excluded) to out[0 .. min(*n_out, cap)). */
uint32_t wcb_generate_tokens(uint32_t handle, const uint32_t* prompt, size_t n, const wcb_gen_config* cfg,
                             uint32_t* out, size_t cap, size_t* n_out);

/* Data-parallel serving: n_seq independent generate() runs through one replica
 * (each sequence has its own KV cache and sampler), each result equal to that
 * sequence's wcb_generate_tokens result. prompts holds the n_seq prompts back
 * to back with lengths lens[]; out is n_seq x cap; n_out receives n_seq counts.
 * On a model loaded with max_batch > 1 the sequences are prefilled one by one
 * into their own KV slots, then their decode steps run together,
 * min(max_batch, 32) sequences per batched step (the weights are read once per
 * step for all of them); otherwise the sequences run one after the other. In a
 * sampled config every sequence draws from the config's seed, as its own
 * generate() does; the batched step's logits are rounded differently from the
 * single-sequence step's, so a sampled sequence can leave its single-sequence
 * tokens where a draw falls within that rounding of a boundary.
 * Replaces the reference's one-sequence-at-a-time serving loop
 * (Model::generate, crates/wasm-chord-runtime/src/transformer/model.rs:1322). */
uint32_t wcb_generate_batch(uint32_t handle, const uint32_t* prompts, const size_t* lens, size_t n_seq,
                            const wcb_gen_config* cfg, uint32_t* out, size_t cap, size_t* n_out);

/* KV slots of one batched decode step (1: no batched path) and the kernels one
 * batched step launches (0 before the first batched wcb_generate_batch). */
uint32_t wcb_batch_info(uint32_t handle, uint32_t* slots, uint32_t* launches_per_step);

/* Streaming generation, the token-id form of the reference's wasmchord_infer /
 * wasmchord_next_token / wasmchord_close_stream (abi.rs:119-200, placeholders
 * there). wcb_infer starts generate()'s loop on a model (clears its KV cache,
 * prefills, samples the first token) and returns a stream handle > 0; starting
 * another generation on the same model invalidates earlier streams. */
uint32_t wcb_infer(uint32_t handle, const uint32_t* prompt, size_t n, const wcb_gen_config* cfg,
                   uint32_t* out_stream);

/* Writes up to max_tokens next generated ids to out (host), running decode
 * steps on the device as needed (greedy decoding runs them back to back without
 * a host round trip); *finished = 1 once EOS or max_tokens has ended the
 * sequence and every token was returned. A KV overflow is reported (code 4) on
 * the call after the last token produced before it. */
uint32_t wcb_next_tokens(uint32_t stream, size_t max_tokens, uint32_t* out, size_t* n_out, uint32_t* finished);

/* One token: returns 1 with *out_token set, -1 at the end, -2 on error
 * (wasmchord_next_token's convention, abi.rs:155-190). */
int32_t wcb_next_token(uint32_t stream, uint32_t* out_token);

uint32_t wcb_close_stream(uint32_t stream);

/* Kernels one greedy decode step launches (for launch accounting). */
uint32_t wcb_model_launches_per_step(uint32_t handle, uint32_t* out);

/* LogitsProcessor (sampling.rs:29-264) over host logits: with_params(seed, T,
 * top_p, top_k, repetition_penalty) -> sampler handle; sample() mutates
 * logits in place (repetition penalty) and records the token. Each sampled
 * (temperature > 0) token takes the next u32 of rand 0.9's
 * StdRng::seed_from_u64(seed) stream, as the reference's sampler does; the
 * device samplers of wcb_generate_* draw from the same stream. */
uint32_t wcb_sampler_new(const wcb_gen_config* cfg, uint32_t* out_sampler);
uint32_t wcb_sampler_sample(uint32_t sampler, float* logits, size_t n, uint32_t* out_token);
uint32_t wcb_sampler_free(uint32_t sampler);
/* The distribution the last sampled (temperature > 0) wcb_sampler_sample drew
 * from: n probabilities (compute_probabilities, top-k, top-p and the
 * renormalisation of sampling.rs:106-229), zero outside the kept candidates. */
uint32_t wcb_sampler_probs(uint32_t sampler, float* out, size_t n);

/* Last error message of the calling thread (wasmchord_last_error, abi.rs:209-222):
 * NUL-terminated, returns bytes copied excluding the NUL. */
size_t wcb_last_error(char* buf, size_t len);

/* Library version string (wasmchord_version, abi.rs:225-228). */
const char* wcb_version(void);

/* ---- Tokenizer (crates/wasm-chord-core/src/tokenizer.rs) and generate(&str) ----
 * wcb_tokenizer_load: Tokenizer::from_gguf (tokenizer.rs:82-147) from a GGUF file's
 * tokenizer.ggml.tokens / tokenizer.ggml.merges / *_token_id metadata; a handle > 0.
 * wcb_tokenize: Tokenizer::encode (tokenizer.rs:207-311): NUL-terminated UTF-8 text
 * (other bytes: WCB_ERR_INVALID_ARGUMENT), BOS first when add_special; *n_out = the
 * id count, min(cap, *n_out) ids written.
 * wcb_detokenize: Tokenizer::decode (tokenizer.rs:353-395): *n_out = the text's byte
 * length; out receives it NUL-terminated, truncated to cap - 1 bytes.
 * wcb_generate_text: Model::generate(prompt, tokenizer, config) (model.rs:1322-1415):
 * encode with BOS, greedy or sampled decoding ended by max_tokens or the tokenizer's
 * EOS (cfg->eos_id is ignored), the prompt and the generated ids decoded together
 * without special tokens; out as for wcb_detokenize. */
uint32_t wcb_tokenizer_load(const char* gguf_path, uint32_t* out_handle);
uint32_t wcb_tokenizer_free(uint32_t tokenizer);
uint32_t wcb_tokenizer_info(uint32_t tokenizer, uint32_t* vocab_size, uint32_t* bos, uint32_t* eos, uint32_t* unk);
/* Tokenizer::set_add_bos_token / set_add_eos_token (tokenizer.rs:417-425) */
uint32_t wcb_tokenizer_set_special(uint32_t tokenizer, uint32_t add_bos, uint32_t add_eos);
uint32_t wcb_tokenize(uint32_t tokenizer, const char* text, uint32_t add_special, uint32_t* out, size_t cap,
                      size_t* n_out);
uint32_t wcb_detokenize(uint32_t tokenizer, const uint32_t* ids, size_t n, uint32_t skip_special, char* out,
                        size_t cap, size_t* n_out);
uint32_t wcb_generate_text(uint32_t model, uint32_t tokenizer, const char* prompt, const wcb_gen_config* cfg,
                           char* out, size_t cap, size_t* n_out);

/* A fresh tensor-parallel group id (ncclGetUniqueId) for wcb_load_opts.tp_id:
 * one rank creates it and the caller hands the same 128 bytes to every rank.
 * No counterpart in the reference. */
uint32_t wcb_tp_id(uint8_t out[128]);

/* Tensor parallelism, decode steps without NCCL: each rank exports the CUDA IPC
 * handle (64 bytes) of its receive buffer, the caller gathers them in rank order
 * and hands all of them to every rank; decode steps (and one-token forwards) then
 * run as one kernel launch per rank that writes its attn-out / ffn-down partial
 * sums and its argmax key straight into every rank's buffer over NVLink and sums
 * them in rank order, every wait bounded by wcb_load_opts.wait_ms (prefill keeps
 * the NCCL all-reduce). No counterpart in the reference. */
uint32_t wcb_model_tp_handle(uint32_t h, uint8_t out[64]);
uint32_t wcb_model_tp_connect(uint32_t h, const uint8_t* handles, uint32_t n_ranks);

/* Tensor parallelism, failure handling: abandons this rank's group after the
 * caller's own failure detector (a heartbeat, a store) found another rank gone.
 * Aborts the NCCL communicator (ncclCommAbort), which also ends a collective
 * still waiting for that rank; every later call on the model then fails with
 * WCB_ERR_BACKEND_UNSUPPORTED, and wcb_model_free releases it without waiting
 * for the other ranks. The one call that may run while another call on the
 * same handle is in progress. A bounded device wait that expires (wait_ms)
 * fails the group the same way. No counterpart in the reference. */
uint32_t wcb_model_tp_abort(uint32_t h);

/* ---- kernel-level entry points (device pointers, caller's stream) ----------
 * No counterpart in the reference's public API: they expose the hot kernels
 * (the reference's quant.rs dequantisers and gemm.rs matmul_transposed) for
 * parity tests and microbenchmarks. `stream` is a cudaStream_t (NULL = legacy
 * default stream). All return after enqueueing; errors are launch errors. */

/* dequantize_q4_k / dequantize_q6_k (quant.rs:58-115, :206-261) over nblocks raw
 * blocks (144 / 210 bytes each, packed) into nblocks*256 floats. Bit-exact. */
uint32_t wcb_dequant_dev(const void* blocks, uint32_t dtype, size_t nblocks, float* out, void* stream);

/* Q6_K blocks are 210 bytes, so they cannot be read with 16-byte loads in
 * place; the device layout pads each block to 224 bytes (bytes 210..223 zero,
 * the first 210 unchanged). Repacks nblocks packed blocks into that layout. */
uint32_t wcb_repack_q6k_dev(const void* packed, size_t nblocks, void* padded, void* stream);

/* y[m][n] = sum_k x[m][k] * W[n][k] (matmul_transposed, gemm.rs:83-143) with W
 * an [n, k] tensor in device layout: raw Q4_K blocks (dtype WCB_DTYPE_Q4_K) or
 * padded Q6_K blocks (WCB_DTYPE_Q6_K, see wcb_repack_q6k_dev). x is [m][k] and
 * y is [m][n], f32, row-major. k % 256 == 0, n % 4 == 0, 1 <= m <= 4096; w and
 * x 16-byte aligned. m <= 4 runs the dp4a GEMV, 5 <= m <= 32 the batched decode
 * GEMM (tcgen05, one launch), larger m the tcgen05 prefill GEMM. */
uint32_t wcb_gemv_dev(const void* w, uint32_t dtype, size_t n, size_t k, const float* x, size_t m, float* y,
                      void* stream);

/* compute_attention (attention.rs:332-435, with repeat_kv :297-322) for n_tokens
 * query tokens on device buffers: q [n_tokens][n_heads][head_dim] (after RoPE),
 * K / V caches [n_kv_heads][max_seq][head_dim] f32 holding kv_len keys, out
 * [n_tokens][n_heads][head_dim]. Query t attends to keys j < kv_len with
 * j <= position + t, scores (q.k) / sqrt(head_dim), softmax, weighted sum of V.
 * head_dim 64 or 128, <= 16 query heads per kv head, n_tokens <= kv_len <= max_seq.
 * A single-token call splits the keys over up to 64 CTAs whose partial results
 * are merged in device scratch this library allocates once per device and
 * reuses; calls that overlap on the GPU race on that scratch. */
uint32_t wcb_attention_dev(const float* q, const float* k_cache, const float* v_cache, float* out, uint32_t n_tokens,
                           uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t max_seq,
                           uint32_t kv_len, uint32_t position, void* stream);

/* The same attention as wcb_attention_dev, for callers that cannot allocate
 * GPU memory once they are running (a host whose device memory is already
 * handed to its own pool, or a serving loop that must not stall its other
 * streams on the device-wide synchronisation of cudaMalloc / cudaFree). No
 * counterpart in the reference. Allocates nothing: the scratch is a fixed
 * 4 MiB array inside the library, which every GPU that loads the library keeps
 * until exit. A call needing more (n_heads * splits * (head_dim + 2) floats for
 * one query token, splits <= 64, plus 4 bytes per query token and kv head)
 * fails with WCB_ERR_INVALID_ARGUMENT. The first call on each device looks up
 * the array's device address; make that first call before any stream capture.
 * All calls share the array: calls that overlap on the GPU race. */
uint32_t wcb_attention_dev_noalloc(const float* q, const float* k_cache, const float* v_cache, float* out,
                                   uint32_t n_tokens, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                                   uint32_t max_seq, uint32_t kv_len, uint32_t position, void* stream);

/* Device stream a model handle launches on (a cudaStream_t), for callers that
 * time or order work against it. */
uint32_t wcb_model_stream(uint32_t handle, void** out_stream);

#ifdef __cplusplus
}
#endif

#endif /* WCB_H */
