/*
 * fl_kernels.h — launch parameters and host launchers of the device kernels.
 * (Internal to libfoundry_cuda.so; the public ABI is include/foundry_cuda.h.)
 */
#ifndef FL_KERNELS_H
#define FL_KERNELS_H

#include <cuda_runtime.h>
#include <stdint.h>

#define FL_MV_MAX_SEG 3
#define FL_TP_MAX 8        /* ranks of one tensor-parallel group */
#define FL_MV_WARPS 8
#define FL_MV_THREADS (FL_MV_WARPS * 32)

/* Input transforms of the matvec prologue (the op that produced the vector in
 * the reference, fused in front of LinearProjection). */
enum {
    FL_IN_PLAIN = 0,        /* x as is; |x| <= *absmax */
    FL_IN_RMSNORM = 1,      /* TensorOperations.RmsNorm(x, w, eps) */
    FL_IN_GEMMA_NORM = 2,   /* TensorOperations.GemmaRmsNorm(x, w) */
    FL_IN_GEMMA_RESID = 3,  /* x' = x + GemmaRmsNorm(pend, pend_w) (stored), then GemmaRmsNorm(x', w) */
};

/* Epilogues (the op that consumed LinearProjection's output). */
enum {
    FL_EPI_STORE = 0,   /* y[row] = v (+ bias) */
    FL_EPI_RESID = 1,   /* y[row] += v  (TensorPrimitives.Add(_x, _xNorm, _x)) */
    FL_EPI_QKV = 2,     /* bias, RoPE, q store, K/V cache append */
    FL_EPI_GLU = 3,     /* act = silu|gelu(gate) * up over interleaved gate/up rows */
    FL_EPI_LOGITS = 4,  /* logits (+ final softcap) and greedy argmax */
};

struct FlMvSeg {
    const uint8_t* w;    /* repacked units of this segment */
    const float* bias;   /* per-row bias (Qwen2) or NULL */
    int32_t fmt, expanded, unit_bytes, n_tiles;
    int32_t tile0;       /* first global tile of the segment */
    int32_t rows;        /* logical rows */
};

struct FlMvArgs {
    FlMvSeg seg[FL_MV_MAX_SEG];
    int32_t n_seg, n_tiles, n_kb, K;
    int32_t slot_bytes, n_slots;   /* per-warp ring */
    /* prologue */
    int32_t in_mode;
    const float* x;
    const float* norm_w;
    float eps;
    const float* pend;
    const float* pend_w;
    float* resid_out;
    const float* absmax;           /* FL_IN_PLAIN bound on |x| */
    /* The rows of the row-parallel projection before this one (Wo, down), as
     * 8-byte words (float bits, exchange tag) in this rank's receive slots,
     * parts[q * part_stride + i] = rank q's partial row i for q < tp_parts
     * (one slot on one GPU): the prologue waits for every word of the
     * exchange's tag and sums them in rank order: FL_IN_RMSNORM x' = x + sum
     * (CTA 0 stores x' in resid_out), FL_IN_GEMMA_RESID pend = sum.  No grid
     * barrier precedes such a phase: the tags are its synchronization.
     * tp_parts = 0: off. */
    int32_t tp_parts, part_stride;
    const unsigned long long* parts;
    /* epilogue */
    int32_t epi;
    float* y;
    int32_t rows_total;
    /* QKV */
    int32_t q_rows, kv_rows, head_dim;
    const float* rope_cs;          /* [max_ctx][head_dim/2][2] cos, sin */
    const int32_t* pos;            /* device position */
    float* q_out;
    float* k_cache;
    float* v_cache;
    /* GLU */
    int32_t act_gelu;
    float* act_out;
    float* act_absmax;
    /* logits */
    float softcap;
    float* cta_best;               /* [grid][2]: value, index bits */
    int32_t* counter;
    int32_t* argmax_out;
    int* err;
    /* tensor parallelism: the LOGITS epilogue writes tp_out[q] = rank q's
     * full logits, rows offset by tp_row0 (the argmax index is global too);
     * the STORE epilogue of a row-parallel projection writes its rows as
     * (float bits, tag) words to tp_out[q] = this rank's receive slot of rank
     * q (q < tp_n; tp_n = 1 on one GPU), tag = the step's exchange count
     * before it + push_x.  tp_n = 0: off. */
    int32_t tp_n, tp_row0, push_x;
    float* tp_out[FL_TP_MAX];
};

/* Dynamic shared memory of a matvec launch. */
size_t fl_mv_smem_bytes(const FlMvArgs& a);
/* Shared memory of a launch without its weight ring (x encoding, barriers,
 * reduction slots) for k-blocks n_kb. */
size_t fl_mv_fixed_smem_bytes(int n_kb);
/* Opts the matvec kernels into large dynamic shared memory on the current
 * device (call before stream capture). */
cudaError_t fl_mv_configure();
cudaError_t fl_launch_matvec(const FlMvArgs& a, int grid, cudaStream_t st, bool pdl);
/* Sizes the per-warp weight ring of a standalone launch (slot = largest unit). */
void fl_mv_ring_config(FlMvArgs& a);

/* Embedding row (bit-exact dequant of token_embd row `token`). */
struct FlEmbedArgs {
    const uint8_t* raw;     /* raw GGUF bytes of token_embd.weight */
    int32_t ggml_type, hidden, vocab;
    const int32_t* token;   /* device token id */
    float* x;
    float* zero_buf;        /* absmax slots cleared each step */
    int32_t zero_n;
    int* err;
};

/* Split-K decode attention over the F32 KV cache. */
struct FlAttnArgs {
    const float* q;              /* [n_heads*head_dim] after RoPE */
    const float* k_cache;        /* [max_ctx][kv_dim] */
    const float* v_cache;
    float* out;                  /* [n_heads*head_dim] */
    float* out_absmax;
    float* part;                 /* [n_kv][n_split][grp][head_dim + 2] */
    int32_t* counter;            /* [n_kv] */
    const int32_t* pos;
    int32_t n_heads, n_kv, head_dim, n_split, window;
    float scale, softcap;
    int* err;
};

/* ── the persistent token kernel (fl_token.cu) ─────────────────────────── */
#define FL_TK_WARPS 16
#ifndef FL_TK_MAX_SLOTS
#define FL_TK_MAX_SLOTS 2        /* ring slots per warp (fewer if shared memory is short) */
#endif
#define FL_TK_MAX_TILES 256      /* 16-row tiles of one matvec phase per CTA */

/* FL_PH_ATTN writes per-split partials; FL_PH_ATTN_COMBINE merges them (same args). */
enum { FL_PH_EMBED = 0, FL_PH_MATVEC = 1, FL_PH_ATTN = 2, FL_PH_ATTN_COMBINE = 3 };

struct FlPhase {
    int32_t kind;
    int32_t xk; /* > 0: this phase reads row exchange xk (1-based) of the step and has no grid barrier before it */
    FlMvArgs mv;
    FlAttnArgs at;
    FlEmbedArgs em;
};

/* A rank's exchange region (one device allocation, mapped by every peer):
 * [FL_TP_MAX] int flags written by peers (epochs), [FL_TP_MAX][2] floats of
 * argmax candidates, [2][FL_TP_MAX][recv_n] 8-byte receive words (rank r
 * pushes its rows of exchange x into [(x - 1) & 1][r] of every rank),
 * [vocab] logits.  On one GPU a session keeps just the [2][1][recv_n] words. */
#define FL_TP_FLAGS_OFF 0
#define FL_TP_BEST_OFF 128
#define FL_TP_RECV_OFF 256

/* What the weight stream needs of one matvec phase, in one 64-byte line. */
struct __align__(64) FlFeedPhase {
    int32_t n_kb, n_tiles, n_seg, pad;
    int32_t tile0[FL_MV_MAX_SEG];
    int32_t unit_bytes[FL_MV_MAX_SEG];
    const uint8_t* w[FL_MV_MAX_SEG];
};

struct FlTokenArgs {
    const FlPhase* phases;       /* device array */
    const FlFeedPhase* feed;     /* [n_feed] the matvec phases, in order */
    int32_t n_feed;
    int32_t n_phases;
    int32_t n_slots, slot_bytes; /* weight ring */
    size_t scratch_bytes;        /* x encoding / attention scratch */
    int32_t* bar;                /* grid barrier counter, zeroed before each launch */
    int* err;
    uint64_t* timestamps;        /* [n_phases + 1] globaltimer at each phase start, CTA 0 */
    uint64_t* cta_done;          /* [n_phases][grid] globaltimer when each CTA finished the phase, or NULL */
    uint64_t* detail;            /* CTA 0, or NULL: [n_phases][warps][4] (units done: globaltimer, cycles
                                    waiting for weights, waits, units) then [n_phases] prologue done */
    /* device-resident decode loop */
    int32_t advance;
    int32_t* token;
    int32_t* pos;
    int32_t* out_tokens;
    int32_t* step;
    /* tensor parallelism (tp_size 1 = off) */
    int32_t tp_size, tp_rank;
    int32_t tp_n_exchanges;      /* flag epochs per step: the argmax exchange */
    int32_t tp_recv_n;           /* floats per receive slot */
    int32_t* tp_epoch;           /* device counters: [0] flag epochs, [1] row exchanges of earlier steps
                                    (the exchange tags; kept on one GPU too) */
    int32_t tp_rows_per_step;    /* row exchanges per step (2 per layer) */
    uint8_t* tp_peer[FL_TP_MAX]; /* every rank's exchange region (this rank's too) */
};

/* The instance for (head_dim, query heads per kv head), or NULL when none is
 * built (head_dim 64/128/256, group <= 8; <= 4 for head_dim 256). */
const void* fl_token_kernel_ptr(int head_dim, int group);
size_t fl_token_smem_bytes(int n_slots, int slot_bytes, size_t scratch_bytes, int n_feed);
/* Opts the instance into the largest dynamic shared memory (before capture). */
cudaError_t fl_token_configure(const void* kernel, int* max_dyn_smem);
cudaError_t fl_launch_token(const void* kernel, const FlTokenArgs& ta, int grid, size_t smem, cudaStream_t st);

/* ── the prompt path (fl_prefill.cu) ───────────────────────────────────── */
#include <cuda_fp16.h>
/* split-fp16 operands: [n x 3K] per matrix, activations [lo | hi | hi], weights [hi | lo | hi] (see fl_prefill.cu) */
#define FL_PF_WSCALE 256.0f
cudaError_t fl_launch_dequant_split(int32_t type, const uint8_t* raw, int rows, int cols, __half* dst, cudaStream_t st,
                                    int layout = 0, int* err = nullptr); /* 0: [hi | lo | hi] rows, 1: [hi | lo] rows */
cudaError_t fl_launch_embed_rows(int32_t type, const uint8_t* raw, const int32_t* tokens, int n, int h, int vocab,
                                 float* x, int* err, cudaStream_t st);
cudaError_t fl_launch_rows_norm(float* x, const float* y, const float* post_w, const float* w, int n, int h, float eps,
                                int gemma, __half* out, cudaStream_t st, int stack = 0,
                                const float* y_lo = nullptr, int* err = nullptr); /* y_lo: a second half added to y */
cudaError_t fl_launch_rope_kv(const float* qkv, const float* bq, const float* bk, const float* bv, const float* rope_cs,
                              int start_pos, int n, int qd, int kvd, int hd, float* q_out, float* k_cache,
                              float* v_cache, cudaStream_t st);
/* batched decode (fl_forward_batch): row b at position row_pos[b] of cache slot row_slot[b] */
cudaError_t fl_launch_rope_kv_rows(const float* qkv, const float* bq, const float* bk, const float* bv,
                                   const float* rope_cs, const int* row_pos, const int* row_slot, size_t slot_stride,
                                   int n, int qd, int kvd, int hd, float* q_out, float* k_cache, float* v_cache,
                                   cudaStream_t st, const float* qkv_lo = nullptr);
cudaError_t fl_launch_batch_attn(const float* q, const float* k_cache, const float* v_cache, const int* row_pos,
                                 const int* row_slot, size_t slot_stride, int B, int nh, int nkv, int hd, int window,
                                 float scale, float softcap, __half* out, cudaStream_t st, int stack = 0,
                                 int* err = nullptr);
cudaError_t fl_launch_softcap_rows(float* x, size_t n, float cap, cudaStream_t st);
cudaError_t fl_launch_add_halves(const float* p, int B, int N, float* y, cudaStream_t st);
cudaError_t fl_launch_argmax_rows(const float* x, int rows, int n, int* out, cudaStream_t st);
/* tensor-parallel prefill: every rank's partial slot and flag array (device
 * addresses, own and peers'), summed in rank order into y once all ranks
 * have raised their flag to epoch */
cudaError_t fl_launch_tp_prefill_reduce(const float* const* slots, int* const* flags, int T, int rank, int epoch,
                                        size_t count, float* y, int* err, cudaStream_t st);
cudaError_t fl_launch_attn_q_split(const float* q, int n, int nh, int nkv, int hd, __half* qs, cudaStream_t st,
                                   int* err = nullptr);
cudaError_t fl_launch_attn_kv_split(const float* kc, const float* vc, int nk, int nkp, int kvd, int hd, __half* ks,
                                    __half* vt, cudaStream_t st, int* err = nullptr);
cudaError_t fl_launch_attn_softmax(const float* S, int rows, int n, int grp, int nkp, int start, int window, float scale,
                                   float softcap, __half* P, cudaStream_t st);
cudaError_t fl_launch_attn_out(const float* O, int n, int nh, int nkv, int hd, __half* act, cudaStream_t st,
                               int* err = nullptr);
cudaError_t fl_launch_glu(const float* g, int n, int F, int gelu, __half* act, cudaStream_t st, int stack = 0,
                          const float* g_lo = nullptr, int* err = nullptr);

/* ── the tcgen05 GEMM (fl_tc_gemm.cu) ──────────────────────────────────────
 * Y[b][n][m] = alpha * sum_k A[b][m][k] * B[b][n][k] (+ beta * Y[b][n][m]),
 * A and B fp16 K-major (row strides lda / ldb elements, 16-byte aligned rows),
 * Y fp32.  With batch > 1, batch b's rows start at row b * a_batch_rows of A
 * and b * b_batch_rows of B, and at Y + b * y_batch. */
struct FlTcGemm {
    int M, N, K, batch;
    int a_batch_rows, b_batch_rows;
    float* Y;
    long long ldy, y_batch;
    float alpha, beta;
    int* err;
    /* ksplit > 1: each output tile's K range in ksplit parts (more CTAs for
     * few tiles); part holds ksplit * batch * N * M floats, summed in split
     * order by a second kernel (deterministic) */
    int ksplit = 1;
    float* part = nullptr;
    /* causal attention of a prompt chunk, B rows = c_grp query rows per token
     * of tokens c_start..: 1 = A rows are keys, tiles past every key a B row
     * may see are skipped (never written); 2 = K is c_seg segments of
     * c_seglen keys (a multiple of 64), each cut to the keys a B row may see
     * (the rest multiply zeros) */
    int causal = 0, c_grp = 1, c_start = 0, c_seg = 0, c_seglen = 0;
};
cudaError_t fl_tc_gemm(const __half* A, long long lda, const __half* B, long long ldb, const FlTcGemm& p,
                       cudaStream_t st);
size_t fl_tc_gemm_smem_bytes(int bn);

/* Bit-exact block dequantization (fl_dequant). */
cudaError_t fl_launch_dequant(int32_t ggml_type, const uint8_t* src, int64_t n_blocks, float* dst, cudaStream_t st);

/* Top-k of a logits vector: k largest (value desc, index asc). */
cudaError_t fl_launch_topk(const float* logits, int32_t n, int32_t k, int32_t* ids, float* vals, uint8_t* scratch,
                           size_t scratch_bytes, cudaStream_t st);
size_t fl_topk_scratch_bytes(int32_t n, int32_t k);
/* sampling (fl_sample.cu) on a working copy w of the logits */
cudaError_t fl_launch_sample_penalty(float* w, const int2* pairs, int n_pairs, float penalty, cudaStream_t st);
cudaError_t fl_launch_sample_scale(float* w, int n, float inv, cudaStream_t st);
cudaError_t fl_launch_sample_topk_mask(float* w, int n, const float* vals, int k, cudaStream_t st);
cudaError_t fl_launch_sample_finish(float* w, int n, int greedy, float top_p, float u, int* token, cudaStream_t st);
/* fl_launch_topk on the file-scope scratch of fl_topk_device (n <= FL_TOPK_DEVICE_MAX_N). */
cudaError_t fl_launch_topk_static(const float* logits, int32_t n, int32_t k, int32_t* ids, float* vals,
                                  cudaStream_t st);

#endif
