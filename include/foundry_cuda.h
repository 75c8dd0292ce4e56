/*
 * foundry_cuda.h — C ABI of the B200 token-loop backend for DotNetFoundryLLM.
 *
 * Plain C: opaque handles, pointers and sizes; no CUDA or torch types.  The
 * C# side binds these with [LibraryImport] in a CudaForwardPass : IForwardPass.
 *
 * Each entry point names the reference interface it replaces (paths inside
 * justinamiller/DotNetFoundryLLM v1.0.0).
 *
 * Error convention: every int-returning call returns FL_OK (0) or one of the
 * FL_ERR_* codes below, and fl_last_error() returns the message of the last
 * failure on the calling thread.  The C# wrapper maps the codes onto the
 * exception types the reference throws (ArgumentOutOfRangeException for a bad
 * token id, NotSupportedException for an unknown tensor type, ...).
 */
#ifndef FOUNDRY_CUDA_H
#define FOUNDRY_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FL_ABI_VERSION 1

#define FL_OK 0
#define FL_ERR_ARG 1          /* ArgumentException / ArgumentOutOfRangeException */
#define FL_ERR_OOM 2          /* device allocation failed */
#define FL_ERR_CUDA 3         /* CUDA runtime error (message has the name) */
#define FL_ERR_NCCL 4         /* NCCL error */
#define FL_ERR_TIMEOUT 5      /* a bounded device-side wait gave up */
#define FL_ERR_UNSUPPORTED 6  /* NotSupportedException (tensor type, shape) */
#define FL_ERR_STATE 7        /* InvalidOperationException / ObjectDisposedException */

#define FL_ARCH_LLAMA 0       /* LlamaForwardPass.cs */
#define FL_ARCH_MISTRAL 1     /* MistralForwardPass.cs */
#define FL_ARCH_GEMMA2 2      /* Gemma2ForwardPass.cs */
#define FL_ARCH_QWEN2 3       /* Qwen2ForwardPass.cs */

#define FL_KV_F32 0           /* KvCache.cs layout: F32 [max_ctx, kv_dim] per layer */

typedef struct fl_model fl_model;
typedef struct fl_session fl_session;

/* Model hyper-parameters: the union of LlamaConfig.cs, MistralConfig.cs and
 * Gemma2Config.cs as GgufModelLoader.BuildConfig/BuildGemma2/BuildMistral fill
 * them (src/DotNetFoundryLLM.ModelFormats.Gguf/GgufModelLoader.cs:104-334). */
typedef struct fl_model_desc {
    int32_t struct_size;      /* sizeof(fl_model_desc) */
    int32_t arch;             /* FL_ARCH_* (GgufModelLoader.Build :89-102) */
    int32_t n_layers;         /* LayerCount */
    int32_t hidden;           /* HiddenSize */
    int32_t ffn;              /* IntermediateSize */
    int32_t n_heads;          /* NumHeads */
    int32_t n_kv_heads;       /* NumKvHeads */
    int32_t head_dim;         /* HeadDim (Gemma2: HeadDimOverride when set) */
    int32_t vocab;            /* VocabSize */
    int32_t max_ctx;          /* MaxContextLength */
    int32_t bos, eos;         /* BosTokenId, EosTokenId */
    int32_t sliding_window;   /* Mistral/Gemma2 SlidingWindowSize; INT32_MAX = none */
    int32_t rope_scaled;      /* 1 when RopeScalingType is linear|yarn and factor > 0 */
    float rms_eps;            /* TensorOperations.RmsNorm eps (1e-5); Gemma2 uses 1e-6 always */
    float rope_base;          /* RopeBaseFreq */
    float rope_factor;        /* RopeScalingFactor */
    float attn_softcap;       /* Gemma2 AttnLogitSoftcap (0 = off) */
    float final_softcap;      /* Gemma2 FinalLogitSoftcap (0 = off) */
    float attn_scale;         /* 1/sqrt(head_dim), or Gemma2 QueryPreAttnScalar */
    int32_t device;           /* CUDA device ordinal for this rank */
    int32_t tp_rank, tp_size; /* tensor parallelism inside one box (1 = off); see fl_session_tp_connect,
                                 and FL_TP_ALL / fl_init for a group driven from one thread */
    const void* nccl_id;      /* reserved (NULL): ranks connect through fl_session_tp_connect */
} fl_model_desc;

/* Last error message of the calling thread ("" when none). */
const char* fl_last_error(void);
int32_t fl_abi_version(void);

/* Replaces GgufModelLoader's F32 weight assembly (LoadWeights :336-372):
 * creates an empty device model for the given config. */
int fl_model_create(const fl_model_desc* desc, fl_model** out);

/* Replaces GgufModelLoader.LoadTensor (GgufModelLoader.cs:409-418) +
 * Dequantizer.Dequantize (Dequantizer.cs:488-504): takes the RAW GGUF block
 * bytes of one tensor (GgufFile.GetTensorBytes, GgufFile.cs:76-97), copies
 * them before returning (the caller's span may be a reused mmap scratch
 * buffer, GgufFile.cs:94-96) and repacks them into the device layout.  No F32
 * expansion happens.  `name` is the GGUF tensor name (token_embd.weight,
 * blk.N.attn_q.weight, ...); dims are in GGUF order (ne0 = row length). */
int fl_model_upload(fl_model* m, const char* name, int32_t ggml_type, const uint64_t* dims, int32_t ndims,
                    const void* bytes, uint64_t nbytes);

/* Checks that every tensor the forward pass needs is present (the
 * "Required tensor ... not found" check of LoadTensor, GgufModelLoader.cs:
 * 411-412; output.weight falls back to token_embd.weight, :368-369). */
int fl_model_finalize(fl_model* m);

/* Replaces LlamaWeights.Dispose (LlamaWeights.cs:93-105). */
void fl_model_destroy(fl_model* m);

/* Per-request forward-pass state: replaces `new KvCache(layers, maxContext,
 * kvDim)` (LlamaLanguageModel.cs:129) and the scratch arrays each forward
 * pass allocates (LlamaForwardPass.cs:54-62).  The KV cache lives in HBM.
 * max_ctx <= 0 uses the model's MaxContextLength.  max_batch (>= 1) is the
 * number of sequence slots, each with its own KV cache of max_ctx positions;
 * slot 0 is the sequence of fl_forward / fl_decode_greedy / fl_prefill, and
 * fl_prefill_seq / fl_forward_batch address any slot (max_batch > 1 needs
 * tp_size 1). */
int fl_session_create(fl_model* m, int32_t max_ctx, int32_t max_batch, int32_t kv_dtype, fl_session** out);

/* Tensor parallelism (fl_model_desc.tp_size = 2, 4 or 8; one process or
 * thread per GPU, every rank with its own model and session).  No
 * counterpart in the reference, which runs on one CPU.  The shim shards the
 * weights as they are uploaded: attn_q/k/v, ffn_gate/up and output by rows
 * (heads, FFN rows, vocabulary), attn_output and ffn_down by columns.  Ranks
 * exchange partial sums and the argmax through each other's memory over
 * NVLink inside the token kernel.  Before its first step a tensor-parallel
 * session must be connected: every rank gets its FL_TP_HANDLE_BYTES handle,
 * the caller gathers the handles of all ranks in rank order (any host-side
 * channel) and passes the array to every rank's fl_session_tp_connect.
 * Ranks in one process are mapped with peer access, others with CUDA IPC;
 * each rank needs a device of its own (ranks of one process that share one
 * are refused with FL_ERR_ARG).  All
 * ranks must then run the same calls (same tokens and positions) in step;
 * a rank that stops makes the others' next step fail with FL_ERR_TIMEOUT
 * after ~2 s.  Logits (fl_forward) and argmax are the full-vocabulary ones
 * on every rank. */
#define FL_TP_HANDLE_BYTES 64

/* Tensor parallelism driven from one host thread, as the reference calls
 * Forward (LlamaForwardPass.cs:29).  fl_init sets the process's layout: tp
 * ranks on devices[0..tp) (NULL: devices 0..tp-1), distinct, each able to
 * access the others' memory.  A model created with tp_rank = FL_TP_ALL and
 * tp_size = tp is then a group: the shim creates one rank per device, each
 * fl_model_upload shards the same bytes to every rank, and fl_session_create
 * connects the ranks' sessions itself (peer access).  A group session takes
 * the calls of a one-GPU session (fl_forward, fl_decode_greedy, fl_prefill,
 * fl_topk, fl_sample, fl_session_reset, fl_time_*) and runs each on all ranks
 * at once, rank 0 on the calling thread and the others on the session's
 * worker threads; logits, argmax and tokens are rank 0's (the full ones).
 * Without fl_init a group uses devices 0..tp_size-1.  fl_forward_batch,
 * fl_prefill_seq and fl_profile_step are one-GPU calls (FL_ERR_UNSUPPORTED). */
#define FL_TP_ALL (-1)
int fl_init(int32_t tp, const int32_t* devices);
int fl_session_tp_handle(fl_session* s, void* handle);
int fl_session_tp_connect(fl_session* s, const void* handles);

/* Recovery of a tensor-parallel group after a call returned FL_ERR_TIMEOUT
 * (a rank stopped or fell out of step).  No counterpart in the reference,
 * which runs on one CPU.  The ranks' exchange epochs have diverged; this
 * restarts this rank's at zero and clears its KV sequence (slot 0).  Every
 * rank calls it once no call is in flight on any rank, and the caller
 * synchronizes the ranks (a host barrier) before and after it; the next call
 * then starts a new sequence at position 0.  A group session (FL_TP_ALL)
 * resets all of its ranks. */
int fl_session_tp_reset(fl_session* s);

/* KvCache.Clear (KvCache.cs:138-144) of one sequence slot. */
int fl_session_reset(fl_session* s, int32_t seq_slot);

/* Batched decode.  No counterpart in the reference, which runs one
 * LlamaLanguageModel.GenerateAsync per request (its BatchCompletion sample is
 * a stub, samples/BatchCompletion/Program.cs:1): one step of `batch`
 * sequences at once, row b being token tokens[b] at position positions[b] of
 * the sequence in slot seq_slots[b] (distinct slots; a position may not skip
 * cached positions; a smaller one rewinds that slot, as IKvCache does).  The
 * values are those of `batch` separate Forward calls.  logits (batch x vocab)
 * and argmax (batch) are host pointers, either may be NULL.  The projections
 * and the LM head run as split-fp16 tensor-core GEMMs over all rows (the
 * prompt path's arithmetic); the weights are dequantized once per session into
 * a cached split layout (6 bytes per weight) when device memory allows, else
 * at every step.  fl_prefill_seq is fl_prefill into a given slot. */
int fl_prefill_seq(fl_session* s, int32_t seq_slot, const int32_t* tokens, int32_t n, int32_t start_pos);
int fl_forward_batch(fl_session* s, int32_t batch, const int32_t* tokens, const int32_t* positions,
                     const int32_t* seq_slots, float* logits, int32_t* argmax);

/* IForwardPass.Forward(tokenId, position, kvCache) (IForwardPass.cs:8-15,
 * LlamaForwardPass.cs:82-130 and the Mistral/Gemma2/Qwen2 copies), plus the
 * greedy sampler (GreedySampler.cs:17 / SamplerPipeline.cs:79-82).
 * K/V for `position` are written into the device cache; attention covers
 * [max(0, position+1-window), position+1).  position must be <= the number of
 * cached positions (a smaller value rewinds).  logits (vocab floats, the
 * IForwardPass.Logits span) and argmax (TensorPrimitives.IndexOfMax, first
 * maximum) are copied to host memory when the pointers are non-NULL. */
int fl_forward(fl_session* s, int32_t token, int32_t position, float* logits, int32_t* argmax);

/* The prompt path: feeds tokens[0..n) at positions start_pos.. into the KV
 * cache, all tokens of a chunk (up to 2048) through one layer at a time.
 * Replaces the prefill loop of LlamaLanguageModel.GenerateAsync
 * (LlamaLanguageModel.cs:133-137: Forward for every prompt token but the
 * last, logits ignored); the last prompt token then goes through fl_forward.
 * The projections run as split-fp16 tensor-core GEMMs (every weight,
 * dequantized bit-exactly, and every activation as an fp16 hi + lo pair;
 * the three significant cross products accumulated in fp32); norms, RoPE,
 * attention and the FFN activation in fp32.  start_pos must not skip cached
 * positions.  With tensor parallelism every rank calls it with the same tokens
 * (each computes its heads and FFN rows; the partial sums after attn_output and
 * ffn_down are exchanged over NVLink through the connected exchange regions). */
int fl_prefill(fl_session* s, const int32_t* tokens, int32_t n, int32_t start_pos);

/* Greedy decode of n_steps tokens entirely on the device: step i feeds the
 * argmax of step i-1 (step 0 feeds `token`) at position start_pos + i.  The
 * generated ids are copied to out_tokens (n_steps ints) at the end.  This is
 * the decode loop of LlamaLanguageModel.GenerateAsync (LlamaLanguageModel.cs:
 * 162-216) with Temperature = 0 and no host round trip per token. */
int fl_decode_greedy(fl_session* s, int32_t token, int32_t start_pos, int32_t n_steps, int32_t* out_tokens);

/* TopKSampler.ApplyTopK (TopKSampler.cs:42-71) on the logits of the last
 * forward: the k largest logits (value descending, index ascending) and the
 * threshold (the k-th largest).  Ties at the threshold are what ApplyTopK
 * keeps; ids/vals receive exactly k entries. */
int fl_topk(fl_session* s, int32_t k, int32_t* ids, float* vals, float* threshold);

/* The sampling step of LlamaLanguageModel.GenerateAsync on the device, on the
 * logits of the session's last fl_forward (which may pass NULL logits):
 * ApplyRepetitionPenalty over `generated` (LlamaLanguageModel.cs:183-186,
 * 357-373), then SamplerPipeline.Sample (SamplerPipeline.cs:58-89):
 * temperature 0 → ArgMax; else scale by 1/T, TopKSampler.ApplyTopK (top_k > 0),
 * Softmax, TopPSampler.ApplyTopP (top_p < 1), SampleFromProbabilities with the
 * draw `u`.  The caller draws u from the request's generator (XoshiroRandom.
 * NextFloat, one draw per call with temperature > 0, none at temperature 0), so
 * a seeded request sees the reference's draws.  The device logits are left
 * unchanged.  Errors as SamplerPipeline's constructor: temperature < 0 or top_p
 * outside (0, 1] → FL_ERR_ARG; also repetition_penalty <= 0. */
typedef struct fl_sampler_desc {
    int32_t struct_size;      /* sizeof(fl_sampler_desc) */
    float temperature;        /* GenerationOptions.Temperature */
    int32_t top_k;            /* GenerationOptions.TopK, <= 0 = off */
    float top_p;              /* GenerationOptions.TopP, 1 = off */
    float repetition_penalty; /* GenerationOptions.RepetitionPenalty, 1 = off */
} fl_sampler_desc;
int fl_sample(fl_session* s, const fl_sampler_desc* d, const int32_t* generated, int32_t n_generated, float u,
              int32_t* token);

void fl_session_destroy(fl_session* s);

/* Allocation-free top-k.  No counterpart in the reference: its sampler works
 * on a managed logits array (TopKSampler.ApplyTopK, TopKSampler.cs:42-71);
 * this entry point serves callers that keep logits on the device and must not
 * allocate per call: an engine whose device memory is one arena reserved up
 * front by its own pool (a .NET host's allocator, a framework's caching
 * allocator), where a cudaMalloc/cudaFree per token would synchronize the
 * device and escape the pool's accounting.  Same selection and order as fl_topk (value descending,
 * index ascending): logits, ids and vals are DEVICE pointers (n floats in, k
 * ints and k floats out), enqueued on `stream` (a cudaStream_t; NULL = the
 * legacy default stream) without synchronizing.
 * - Scratch: a file-scope device array of FL_TOPK_DEVICE_MAX_N * 8 bytes
 *   (2 MiB) per device; n > FL_TOPK_DEVICE_MAX_N returns FL_ERR_ARG.  Nothing
 *   in it has to start at zero.  No cudaMalloc, cudaFree or allocating library
 *   call is made.
 * - Every call looks the scratch address up on the current device
 *   (cudaGetSymbolAddress, which allocates nothing), so a device reset in
 *   between is harmless.  The first call on a device also loads the module
 *   there: make that first call outside any stream capture.
 * - All calls on one device share the scratch: calls that overlap in time
 *   (different streams or threads, or a call whose previous kernel has not
 *   finished on another stream) race and may return wrong results. */
#define FL_TOPK_DEVICE_MAX_N 262144
int fl_topk_device(const float* logits, int32_t n, int32_t k, int32_t* ids, float* vals, void* stream);

/* Dequantizer.Dequantize (Dequantizer.cs:488-504) on the device, bit-exact:
 * src is host memory with whole blocks, dst receives the F32 values.
 * Returns FL_ERR_ARG for a length that is not a multiple of the block size or a
 * dst that is too small (the ArgumentException cases), FL_ERR_UNSUPPORTED for
 * a type id outside {0,1,2,8,12,13,14,15,30}. */
int fl_dequant(int32_t ggml_type, const void* src, uint64_t nbytes, float* dst, uint64_t dst_len);

/* One dequant-matvec launch, y = W x, through the same repack and kernel the
 * forward pass uses (LinearProjection, LlamaForwardPass.cs:237-260, over the
 * quantized weights).  W is raw GGUF bytes for rows x cols elements. */
int fl_matvec(int32_t ggml_type, const void* w, uint64_t nbytes, int32_t rows, int32_t cols, const float* x,
              float* y);

/* Test hook: the tensor-core GEMM of the prompt path and of batched decode
 * (tcgen05, fp16 operands, fp32 accumulation), the LinearProjection of
 * LlamaForwardPass.cs:237-260 over a chunk of rows.  Host memory in and out:
 * for each batch b < batch, y[b][n][m] = alpha * sum_k a[b][m][k] * b[b][n][k]
 * + beta * y[b][n][m], with a (fp16 bits) holding batch * a_batch_rows rows
 * of lda elements (M rows when batch is 1), b likewise, y dense
 * [batch][N][M] fp32.  lda and ldb are multiples of 8.
 * ksplit > 1: each output tile's K range split over ksplit work items, their
 * partials summed in split order.  causal (the prompt path's attention, with
 * c_grp B rows per token of tokens c_start..): 1 = a[m] are keys and y[n][m]
 * is left unwritten for every key past the last one token n / c_grp's tile
 * may see (keys 0..c_start + that token); 2 = K is c_seg segments, each cut
 * to those keys (a multiple of 64 long). */
int fl_gemm_f16(const void* a, int64_t lda, const void* b, int64_t ldb, int32_t M, int32_t N, int32_t K,
                int32_t batch, int32_t a_batch_rows, int32_t b_batch_rows, float alpha, float beta, int32_t ksplit,
                int32_t causal, int32_t c_grp, int32_t c_start, int32_t c_seg, float* y);

/* Timing helpers for the benchmark: runs one token step and reads the
 * device timestamps the token kernel takes at every phase boundary; fills
 * ms[class] (time spent in phases of that class) and bytes[class]
 * (algorithmic bytes) for the FL_PROF_* classes, and *launches with the
 * kernels one step launches. */
#define FL_PROF_MATVEC 0
#define FL_PROF_ATTN 1
#define FL_PROF_OTHER 2
#define FL_PROF_STEP 3
#define FL_PROF_N 4
int fl_profile_step(fl_session* s, int32_t token, int32_t position, double* ms, double* bytes, int32_t* launches);

/* Device step time of the captured token graph: runs n_steps greedy steps as
 * in fl_decode_greedy and returns the elapsed device milliseconds (CUDA events
 * on the session stream). */
int fl_time_decode(fl_session* s, int32_t token, int32_t start_pos, int32_t n_steps, float* ms);

/* fl_prefill with its device time: the chunk loop bracketed by CUDA events on
 * the session stream (token upload included), elapsed milliseconds in *ms. */
int fl_time_prefill(fl_session* s, const int32_t* tokens, int32_t n, int32_t start_pos, float* ms);

/* Bytes of weights one decode step reads (the GGUF payload of every matrix,
 * norm and one embedding row): the roofline numerator without the KV term. */
int fl_model_weight_bytes(fl_model* m, double* bytes);

/* Number of kernels the token graph launches per step. */
int fl_session_launches_per_step(fl_session* s, int32_t* n);

#ifdef __cplusplus
}
#endif
#endif
