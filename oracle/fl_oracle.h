/*
 * fl_oracle.h — CPU restatement of DotNetFoundryLLM's token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA path: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg load it.  The product library (libfoundry_cuda.so) never links or calls
 * it, and it is never the thing that is measured as the GPU result.
 *
 * Each function follows one C# method of the reference; the citation
 * (path:line within justinamiller/DotNetFoundryLLM v1.0.0) sits beside it in
 * fl_oracle.c.  Pinning: the dequantizer, HalfToFloat/BFloat16ToFloat,
 * ElementCount, the GGUF header parser and greedy ArgMax are checked against
 * every known-answer vector the reference's own xUnit tests hold
 * (tests/golden/reference_kats.json).  Q6_K/Q8_K, non-zero K-quant blocks
 * and forward-pass logits are not pinned by any reference test; for those the
 * restatement is the golden (parity unpinned: it follows the reference's
 * operation order, and the reference's TensorPrimitives reductions are
 * ISA-dependent, so forward-pass parity is judged by tolerance).
 */
#ifndef FL_ORACLE_H
#define FL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes returned by the oracle (negative = the C# exception type). */
#define OR_OK 0
#define OR_ARGUMENT_EXCEPTION (-1)          /* System.ArgumentException */
#define OR_NOT_SUPPORTED (-2)               /* System.NotSupportedException */
#define OR_ARGUMENT_OUT_OF_RANGE (-3)       /* System.ArgumentOutOfRangeException */
#define OR_INVALID_OPERATION (-4)           /* System.InvalidOperationException */
#define OR_MODEL_LOAD (-5)                  /* DotNetFoundryLLM.Core.ModelLoadException */

/* ── Quantization/Dequantizer.cs ─────────────────────────────────────── */
float or_half_to_float(uint16_t bits);
float or_bf16_to_float(uint16_t bits);
int64_t or_element_count(int tensor_type, int64_t byte_length); /* OR_NOT_SUPPORTED on bad type */
int or_dequantize(int tensor_type, const uint8_t* src, int64_t src_len, float* dst, int64_t dst_len);

/* ── Tensors/TensorOperations.cs ─────────────────────────────────────── */
float or_dot(const float* a, const float* b, int n);
void or_rmsnorm(const float* x, const float* w, float* dst, int n, float eps);
void or_gemma_rmsnorm(const float* x, const float* w, float* dst, int n);
void or_softmax(float* x, int n);
void or_silu(float* x, int n);
void or_gelu(float* x, int n);
void or_softcap(float* x, int n, float cap);
int or_argmax(const float* x, int n);
void or_apply_topk(float* logits, int n, int k);
void or_rope(float* x, float position, const float* inv_freqs, int half);

/* ── Sampling (the Sampling project, Core/XoshiroRandom.cs, Inference) ───── */
void or_xoshiro_seed(uint64_t seed, uint64_t* state4);
uint64_t or_xoshiro_next(uint64_t* state4);
float or_xoshiro_next_float(uint64_t* state4);
void or_apply_repetition_penalty(float* logits, int n, const int* generated, int n_generated, float penalty);
void or_apply_topp(float* probs, int n, float p);
int or_sample_from_probs(const float* probs, int n, float u);
/* SamplerPipeline.Sample on logits (modified in place); u is the pipeline's
 * NextFloat draw (unused when temperature is 0). */
int or_sampler_pipeline(float* logits, int n, float temperature, int top_k, float top_p, float u);

/* ── ModelFormats.Gguf ─────────────────────────────────────────────────── */
typedef struct or_gguf or_gguf;
/* Parses a whole GGUF image held in memory (GgufReader.Parse).  The image
 * must outlive the handle.  Returns NULL and fills err on failure. */
or_gguf* or_gguf_parse(const uint8_t* data, int64_t len, char* err, int errlen);
void or_gguf_free(or_gguf* g);
uint32_t or_gguf_version(const or_gguf* g);
int64_t or_gguf_tensor_count(const or_gguf* g);
int64_t or_gguf_kv_count(const or_gguf* g);
int64_t or_gguf_data_start(const or_gguf* g);
/* Tensor lookup: returns index or -1. */
int64_t or_gguf_find_tensor(const or_gguf* g, const char* name);
int or_gguf_tensor_info(const or_gguf* g, int64_t idx, int* type, int* ndims, uint64_t* dims4,
                        uint64_t* offset, int64_t* nbytes);

/* ── Architectures + Inference (model, KV cache, forward, generate) ──── */
typedef struct or_model or_model;
typedef struct or_session or_session;

/* Loads a model from a GGUF image exactly as GgufModelLoader does
 * (metadata → config, every tensor dequantized to F32 at load time).
 * max_layers < 0 loads every layer; a smaller value loads only the first
 * max_layers blocks (used to time a bounded sample of a large model). */
or_model* or_model_load(const uint8_t* data, int64_t len, int max_layers, char* err, int errlen);
/* lazy = 1: weight matrices stay as the image's raw blocks (the caller keeps
 * `data` alive) and are dequantized row by row where used; same values. */
or_model* or_model_load_ex(const uint8_t* data, int64_t len, int max_layers, int lazy, char* err, int errlen);
void or_model_free(or_model* m);
/* Config readback: arch (0 llama, 1 mistral, 2 gemma2, 3 qwen2), dims[...] */
void or_model_config(const or_model* m, int* arch, int* ints12, float* floats8);

or_session* or_session_create(or_model* m);
void or_session_free(or_session* s);
int or_session_length(const or_session* s);
/* Timing samples only: pretend the cache holds n positions. */
int or_session_fake_length(or_session* s, int n);
/* IForwardPass.Forward: logits copied to logits_out (may be NULL). */
int or_forward(or_session* s, int token, int position, float* logits_out);
/* Runs layers [0, n_layers) of one forward pass only (timing sample). */
int or_forward_layers(or_session* s, int token, int position, int n_layers);
/* LM-head matvec on the current residual stream (timing sample). */
int or_forward_head(or_session* s, float* logits_out);
/* LlamaLanguageModel.GenerateAsync with temperature 0 (greedy). */
int or_generate_greedy(or_model* m, const int* prompt, int n_prompt, int max_tokens,
                       int* out_tokens, float* out_logits /* max_tokens*vocab or NULL */);

void or_set_threads(int n);
int or_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
