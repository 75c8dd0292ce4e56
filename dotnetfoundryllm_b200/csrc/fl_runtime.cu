/*
 * fl_runtime.cu — the C ABI (include/foundry_cuda.h): device model, upload +
 * repack, per-request session with an HBM KV cache, and the token step as one
 * persistent cooperative kernel (fl_token.cu) replayed from a CUDA graph.
 *
 * Reference seam: LlamaLanguageModel takes a Func<IForwardPass> factory and an
 * IDisposable model resource (src/DotNetFoundryLLM.Inference/
 * LlamaLanguageModel.cs:48-80); fl_model is that resource and fl_session +
 * fl_forward the IForwardPass (IForwardPass.cs:8-15).
 */
#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <functional>
#include <thread>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>


#include "../../include/foundry_cuda.h"
#include "fl_kernels.h"
#include "fl_repack.h"

/* ── errors ─────────────────────────────────────────────────────────────── */
static thread_local std::string g_err;

static int fail(int code, const char* fmt, ...)
{
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) {                                                                   \
            if (e_ == cudaErrorMemoryAllocation)                                                   \
                return fail(FL_ERR_OOM, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
            return fail(FL_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
        }                                                                                          \
    } while (0)

extern "C" const char* fl_last_error(void) { return g_err.c_str(); }
extern "C" int32_t fl_abi_version(void) { return FL_ABI_VERSION; }

/* ── device objects ─────────────────────────────────────────────────────── */
struct DevMatrix {
    fl_matrix_layout L;
    uint8_t* d = nullptr;
    bool present = false;
};

/* A matrix's raw GGUF blocks on the device (the prompt path dequantizes them
 * to fp16 for its GEMMs; rows x cols in GGUF row-major order). */
struct RawMatrix {
    uint8_t* d = nullptr;
    int type = -1;
    int rows = 0, cols = 0;
};

struct Layer {
    DevMatrix wq, wk, wv, wo, gate_up, down;
    float *attn_norm = nullptr, *ffn_norm = nullptr, *post_attn_norm = nullptr, *post_ffn_norm = nullptr;
    float *bq = nullptr, *bk = nullptr, *bv = nullptr;
    std::vector<uint8_t> stash;      /* raw bytes of gate or up until its partner arrives */
    int stash_type = -1, stash_is_gate = 0;
    RawMatrix rq, rk, rv, ro, rgate, rup, rdown; /* raw blocks for the prompt path and batched decode */
};

struct fl_model {
    fl_model_desc d;
    int sm_count = 148;
    /* tensor parallelism: this rank's share (T = 1: the whole model) */
    int T = 1, rank = 0;
    int nh_l = 0, nkv_l = 0, qd_l = 0, kvd_l = 0, ffn_l = 0, vocab_l = 0;
    std::vector<Layer> layers;
    uint8_t* emb_raw = nullptr;
    int emb_type = -1;
    int64_t emb_bytes = 0;
    DevMatrix output;
    RawMatrix rout; /* the LM head's raw blocks (one GPU): output.weight, or token_embd when tied */
    float* out_norm = nullptr;
    float* rope_cs = nullptr;
    bool finalized = false;
    std::vector<void*> allocs;
    double weight_bytes = 0;
    /* a tensor-parallel group driven from one host thread (tp_rank FL_TP_ALL):
     * one rank model per device; the fields above stay unused */
    bool group = false;
    std::vector<fl_model*> ranks;
};

struct fl_session {
    fl_model* m = nullptr;
    int max_ctx = 0, cur_len = 0; /* cur_len: the length of slot 0, the token loop's sequence */
    /* sequence slots (max_batch): slot i's K (and V) cache starts slot_stride floats after slot i-1's */
    int n_slots = 1;
    size_t slot_stride = 0;
    std::vector<int> slot_len; /* lengths of slots 1.. */
    cudaStream_t st = nullptr;
    float *xa = nullptr, *xb = nullptr, *q = nullptr, *att = nullptr, *act = nullptr, *o = nullptr, *logits = nullptr;
    float *kc = nullptr, *vc = nullptr;
    float* absmax = nullptr; /* [2*L] attn_out, act */
    int n_absmax = 0;
    int32_t* state = nullptr; /* token, pos, argmax, step, err, head_counter */
    int32_t* attn_counter = nullptr;
    float* attn_part = nullptr;
    /* fl_sample: working copy of the logits (+ the token), (id, count) pairs */
    float* samp_w = nullptr;
    int32_t* samp_tok = nullptr;
    int2* samp_pairs = nullptr;
    size_t samp_pairs_cap = 0;
    float* cta_best = nullptr;
    int32_t* out_tokens = nullptr;
    int32_t* topk_ids = nullptr;
    float* topk_vals = nullptr;
    uint8_t* topk_scratch = nullptr;
    size_t topk_scratch_bytes = 0;
    int32_t* h_state = nullptr; /* pinned */
    cudaGraphExec_t graph = nullptr;
    int launches = 0;
    int attn_split = 1;
    /* the token step: phase list + persistent kernel configuration */
    FlPhase* d_phases = nullptr;
    FlFeedPhase* d_feed = nullptr;
    int n_phases = 0;
    std::vector<int> phase_cls;
    std::vector<double> phase_bytes;
    int32_t* bar = nullptr;
    uint64_t* timestamps = nullptr;
    uint64_t* cta_done = nullptr;
    uint64_t* detail = nullptr;
    FlTokenArgs ta;
    size_t tk_smem = 0;
    int tk_grid = 0;
    const void* tk_kernel = nullptr;
    int max_dyn = 0;
    bool built = false;
    /* tensor parallelism: this rank's exchange region and every rank's, mapped */
    uint8_t* xchg = nullptr;
    size_t xchg_bytes = 0, xchg_logits_off = 0, xchg_pf_off = 0;
    int pf_tp_rows = 0; /* rows of a prompt chunk's partial-sum slot in the exchange region */
    int32_t pf_epoch = 0; /* the prompt path's flag epoch (host copy while it runs) */
    int xchg_recv_n = 0;
    int tp_rows_per_step = 0; /* row exchanges of one token step (2 per layer) */
    int32_t* tp_epoch = nullptr;
    uint8_t* tp_peer[FL_TP_MAX] = {};
    void* tp_opened[FL_TP_MAX] = {};
    /* the prompt path, allocated by the first fl_prefill */
    int pf_cap = 0;
    int32_t* pf_tokens = nullptr;
    float *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_y = nullptr;
    __half *pf_act = nullptr, *pf_w = nullptr;
    /* batched decode (fl_forward_batch): row positions, slots, logits, argmax;
     * the split-fp16 weights cached on the first call when memory allows
     * (per layer qkv, wo, gate/up, down; then the LM head) */
    int32_t *bt_pos = nullptr, *bt_slot = nullptr, *bt_argmax = nullptr;
    float* bt_logits = nullptr;
    float* bt_y2 = nullptr; /* [2 * slots][widest projection] the two output halves of a batched projection */
    float* bt_part = nullptr; /* K-split partial products of a batched projection */
    bool bt_cache_tried = false;
    std::vector<__half*> bt_w;
    /* attention of a chunk: split Q/K/V^T, scores, split probabilities, output */
    int pf_nkmax = 0;
    __half *pf_qs = nullptr, *pf_ks = nullptr, *pf_vt = nullptr, *pf_p = nullptr;
    float *pf_s = nullptr, *pf_o = nullptr;
    std::vector<void*> allocs;
    /* a group session: one connected rank session per device and the worker
     * threads that run ranks 1.. while the caller runs rank 0 */
    bool group = false;
    std::vector<fl_session*> ranks;
    struct RankPool* pool = nullptr;
};

/* ── tensor-parallel groups (defined at the end of this file) ───────────── */
static int group_model_create(const fl_model_desc& d, fl_model** out);
static int group_session_create(fl_model* g, int32_t max_ctx, int32_t max_batch, int32_t kv_dtype, fl_session** out);
static void group_session_destroy(fl_session* s);
static int run_ranks(fl_session* s, const std::function<int(int)>& f);

enum { ST_TOKEN = 0, ST_POS = 1, ST_ARGMAX = 2, ST_STEP = 3, ST_ERR = 4, ST_HEADCNT = 5, ST_N = 8 };

template <typename T>
static int dalloc(std::vector<void*>& list, T** p, size_t bytes)
{
    void* v = nullptr;
    cudaError_t e = cudaMalloc(&v, bytes ? bytes : 16);
    if (e != cudaSuccess) return fail(FL_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    list.push_back(v);
    *p = reinterpret_cast<T*>(v);
    return FL_OK;
}

static int block_elems(int t)
{
    switch (t) {
    case FL_T_F32: case FL_T_F16: case FL_T_BF16: return 1;
    case FL_T_Q4_0: case FL_T_Q8_0: return 32;
    case FL_T_Q4_K: case FL_T_Q5_K: case FL_T_Q6_K: case FL_T_Q8_K: return 256;
    default: return 0;
    }
}
static int block_bytes(int t)
{
    switch (t) {
    case FL_T_F32: return 4;
    case FL_T_F16: case FL_T_BF16: return 2;
    case FL_T_Q4_0: return 18;
    case FL_T_Q8_0: return 34;
    case FL_T_Q4_K: return 144;
    case FL_T_Q5_K: return 176;
    case FL_T_Q6_K: return 210;
    case FL_T_Q8_K: return 292;
    default: return 0;
    }
}

/* ── model ──────────────────────────────────────────────────────────────── */
extern "C" int fl_model_create(const fl_model_desc* desc, fl_model** out)
{
    if (!desc || !out) return fail(FL_ERR_ARG, "null argument");
    if (desc->struct_size != (int32_t)sizeof(fl_model_desc)) return fail(FL_ERR_ARG, "fl_model_desc size mismatch");
    const fl_model_desc& d = *desc;
    if (d.tp_rank == FL_TP_ALL) return group_model_create(d, out);
    if (d.arch < FL_ARCH_LLAMA || d.arch > FL_ARCH_QWEN2) return fail(FL_ERR_UNSUPPORTED, "unknown arch %d", d.arch);
    /* LlamaForwardPass.cs:48-52 */
    if (d.n_kv_heads <= 0 || d.n_heads <= 0 || d.n_kv_heads > d.n_heads || d.n_heads % d.n_kv_heads != 0)
        return fail(FL_ERR_ARG, "Invalid attention head configuration: NumHeads=%d, NumKvHeads=%d.", d.n_heads,
                    d.n_kv_heads);
    if (d.n_layers <= 0 || d.hidden <= 0 || d.ffn <= 0 || d.vocab <= 0 || d.max_ctx <= 0)
        return fail(FL_ERR_ARG, "non-positive dimension");
    if (d.head_dim != 64 && d.head_dim != 128 && d.head_dim != 256)
        return fail(FL_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128, 256)", d.head_dim);
    int grp = d.n_heads / d.n_kv_heads;
    if (grp > 8 || (d.head_dim == 256 && grp > 4)) return fail(FL_ERR_UNSUPPORTED, "GQA group %d", grp);
    if (d.hidden % 32 || d.ffn % 32 || (d.n_heads * d.head_dim) % 32)
        return fail(FL_ERR_UNSUPPORTED, "dimensions must be multiples of 32");
    const int T = d.tp_size < 1 ? 1 : d.tp_size;
    if (T > FL_TP_MAX || (T & (T - 1))) return fail(FL_ERR_UNSUPPORTED, "tp_size %d (1, 2, 4 or 8)", T);
    if (d.tp_rank < 0 || d.tp_rank >= T) return fail(FL_ERR_ARG, "tp_rank %d outside [0, %d)", d.tp_rank, T);
    if (d.n_kv_heads % T || d.ffn % (8 * T) || d.vocab % (16 * T))
        return fail(FL_ERR_UNSUPPORTED, "tp_size %d does not divide the kv heads (%d), FFN rows (%d) or vocabulary (%d)",
                    T, d.n_kv_heads, d.ffn, d.vocab);
    if (cudaSetDevice(d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice(%d) failed", d.device);
    fl_model* m = new fl_model();
    m->d = d;
    m->T = T;
    m->rank = T > 1 ? d.tp_rank : 0;
    m->nh_l = d.n_heads / T;
    m->nkv_l = d.n_kv_heads / T;
    m->qd_l = m->nh_l * d.head_dim;
    m->kvd_l = m->nkv_l * d.head_dim;
    m->ffn_l = d.ffn / T;
    m->vocab_l = d.vocab / T;
    m->layers.resize((size_t)d.n_layers);
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d.device) == cudaSuccess && sms > 0)
        m->sm_count = sms;
    /* RoPE table: theta = pos' * invFreq[i], invFreq[i] = 1/powf(base, 2i/hd)
     * (LlamaForwardPass.cs:64-70, 135-148; TensorOperations.cs:250-260),
     * cos/sin from the C runtime as MathF does on Linux. */
    const int half = d.head_dim / 2;
    std::vector<float> inv((size_t)half), cs((size_t)d.max_ctx * half * 2);
    for (int i = 0; i < half; i++) {
        float ex = (2.0f * (float)i) / (float)d.head_dim;
        inv[(size_t)i] = 1.0f / powf(d.rope_base, ex);
    }
    for (int p = 0; p < d.max_ctx; p++) {
        float pos = d.rope_scaled ? (float)p / d.rope_factor : (float)p;
        for (int i = 0; i < half; i++) {
            float th = pos * inv[(size_t)i];
            cs[((size_t)p * half + i) * 2] = cosf(th);
            cs[((size_t)p * half + i) * 2 + 1] = sinf(th);
        }
    }
    int rc = dalloc(m->allocs, &m->rope_cs, cs.size() * 4);
    if (rc) { delete m; return rc; }
    if (cudaMemcpy(m->rope_cs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        fl_model_destroy(m);
        return fail(FL_ERR_CUDA, "rope table upload failed");
    }
    *out = m;
    return FL_OK;
}

extern "C" void fl_model_destroy(fl_model* m)
{
    if (!m) return;
    if (m->group) {
        for (fl_model* r : m->ranks) fl_model_destroy(r);
        delete m;
        return;
    }
    cudaSetDevice(m->d.device);
    for (void* p : m->allocs) cudaFree(p);
    delete m;
}

/* Dequantizes a small tensor (norm weights, biases) on the device, bit-exact. */
static int upload_vector(fl_model* m, int type, const void* bytes, uint64_t nbytes, int64_t expect, float** out)
{
    int be = block_elems(type), bb = block_bytes(type);
    if (!be) return fail(FL_ERR_UNSUPPORTED, "Tensor type %d is not supported for dequantization.", type);
    if (nbytes % (uint64_t)bb) return fail(FL_ERR_ARG, "tensor byte length is not a multiple of the block size");
    int64_t n = (int64_t)(nbytes / bb) * be;
    if (n != expect) return fail(FL_ERR_ARG, "vector has %lld elements, expected %lld", (long long)n, (long long)expect);
    uint8_t* raw = nullptr;
    float* dst = nullptr;
    int rc = dalloc(m->allocs, &dst, (size_t)expect * 4);
    if (rc) return rc;
    CK(cudaMalloc(&raw, nbytes));
    CK(cudaMemcpy(raw, bytes, nbytes, cudaMemcpyHostToDevice));
    CK(fl_launch_dequant(type, raw, n, dst, 0));
    CK(cudaDeviceSynchronize());
    CK(cudaFree(raw));
    *out = dst;
    m->weight_bytes += (double)nbytes;
    return FL_OK;
}

static int upload_matrix(fl_model* m, int type, int rows, int cols, const uint8_t* raw, const uint8_t* raw2,
                         const int32_t* row_map, DevMatrix* dm, double gguf_bytes)
{
    fl_matrix_layout L;
    int r = fl_layout_for(type, rows, cols, &L);
    if (r == -1) return fail(FL_ERR_UNSUPPORTED, "matrix type %d has no quantized matvec path", type);
    if (r == -2) return fail(FL_ERR_UNSUPPORTED, "matrix row length %d is not a multiple of 32", cols);
    std::vector<uint8_t> host((size_t)L.total_bytes);
    fl_repack(&L, raw, raw2, row_map, host.data(), 0);
    int rc = dalloc(m->allocs, &dm->d, (size_t)L.total_bytes);
    if (rc) return rc;
    CK(cudaMemcpy(dm->d, host.data(), (size_t)L.total_bytes, cudaMemcpyHostToDevice));
    dm->L = L;
    dm->present = true;
    m->weight_bytes += gguf_bytes;
    return FL_OK;
}

/* Tensor parallelism: this rank's rows [r0, r0 + n) of a row-major matrix
 * (whole rows of GGUF blocks), or its columns [c0, c0 + n) of every row
 * (whole blocks: the split must be a multiple of the block length). */
static std::vector<uint8_t> slice_rows(const uint8_t* raw, int type, int cols, int r0, int n)
{
    const size_t rb = (size_t)cols / block_elems(type) * block_bytes(type);
    return std::vector<uint8_t>(raw + (size_t)r0 * rb, raw + (size_t)(r0 + n) * rb);
}

static std::vector<uint8_t> slice_cols(const uint8_t* raw, int type, int rows, int cols, int c0, int n)
{
    const size_t rb = (size_t)cols / block_elems(type) * block_bytes(type);
    const size_t b0 = (size_t)c0 / block_elems(type) * block_bytes(type);
    const size_t nb = (size_t)n / block_elems(type) * block_bytes(type);
    std::vector<uint8_t> out((size_t)rows * nb);
    for (int r = 0; r < rows; r++) memcpy(out.data() + (size_t)r * nb, raw + (size_t)r * rb + b0, nb);
    return out;
}

/* Internal (tests): the slice a rank keeps, rows (dim 0) or columns (dim 1). */
extern "C" int fl_tp_slice(int32_t type, int32_t rows, int32_t cols, int32_t dim, int32_t rank, int32_t T,
                           const void* src, void* dst)
{
    if (!block_elems(type) || T < 1 || rank < 0 || rank >= T) return fail(FL_ERR_ARG, "bad slice request");
    std::vector<uint8_t> v;
    if (dim == 0) {
        if (rows % T) return fail(FL_ERR_ARG, "rows %d not divisible by %d", rows, T);
        v = slice_rows(static_cast<const uint8_t*>(src), type, cols, rank * (rows / T), rows / T);
    } else {
        if (cols % T || (cols / T) % block_elems(type)) return fail(FL_ERR_ARG, "columns %d do not split by %d", cols, T);
        v = slice_cols(static_cast<const uint8_t*>(src), type, rows, cols, rank * (cols / T), cols / T);
    }
    memcpy(dst, v.data(), v.size());
    return FL_OK;
}

static int keep_raw(fl_model* m, RawMatrix* rm, int type, int rows, int cols, const uint8_t* raw, uint64_t nbytes)
{
    int rc = dalloc(m->allocs, &rm->d, nbytes);
    if (rc) return rc;
    CK(cudaMemcpy(rm->d, raw, nbytes, cudaMemcpyHostToDevice));
    rm->type = type;
    rm->rows = rows;
    rm->cols = cols;
    return FL_OK;
}

static bool parse_layer(const char* name, int* layer, std::string* suffix)
{
    if (strncmp(name, "blk.", 4) != 0) return false;
    char* end = nullptr;
    long l = strtol(name + 4, &end, 10);
    if (!end || *end != '.') return false;
    *layer = (int)l;
    *suffix = end + 1;
    return true;
}

extern "C" int fl_model_upload(fl_model* m, const char* name, int32_t type, const uint64_t* dims, int32_t ndims,
                               const void* bytes, uint64_t nbytes)
{
    if (!m || !name || !dims || ndims <= 0 || ndims > 4 || (!bytes && nbytes)) return fail(FL_ERR_ARG, "null argument");
    if (m->group) { /* every rank takes its shard of the same bytes */
        for (fl_model* r : m->ranks) {
            int rc = fl_model_upload(r, name, type, dims, ndims, bytes, nbytes);
            if (rc) return rc;
        }
        return FL_OK;
    }
    if (m->finalized) return fail(FL_ERR_STATE, "model already finalized");
    if (!block_elems(type)) return fail(FL_ERR_UNSUPPORTED, "Tensor type %d is not supported for dequantization.", type);
    if (cudaSetDevice(m->d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    int64_t elems = 1;
    for (int i = 0; i < ndims; i++) elems *= (int64_t)dims[i];
    if (elems % block_elems(type) || (uint64_t)(elems / block_elems(type) * block_bytes(type)) != nbytes)
        return fail(FL_ERR_ARG, "%s: %llu bytes do not match %lld elements of type %d", name,
                    (unsigned long long)nbytes, (long long)elems, type);
    const fl_model_desc& d = m->d;
    const int h = d.hidden, qd = d.n_heads * d.head_dim, kvd = d.n_kv_heads * d.head_dim, f = d.ffn;
    const uint8_t* raw = static_cast<const uint8_t*>(bytes);
    auto mat_shape_ok = [&](int rows, int cols) {
        return ndims >= 2 && (int64_t)dims[0] == cols && elems == (int64_t)rows * cols;
    };
    std::string n(name);
    if (n == "token_embd.weight") {
        if (elems != (int64_t)d.vocab * h) return fail(FL_ERR_ARG, "token_embd.weight has %lld elements", (long long)elems);
        int rc = dalloc(m->allocs, &m->emb_raw, nbytes);
        if (rc) return rc;
        CK(cudaMemcpy(m->emb_raw, raw, nbytes, cudaMemcpyHostToDevice));
        m->emb_type = type;
        m->emb_bytes = (int64_t)nbytes;
        return FL_OK;
    }
    if (n == "output_norm.weight") return upload_vector(m, type, raw, nbytes, h, &m->out_norm);
    const int T = m->T, rk = m->rank;
    if (n == "output.weight") {
        if (!mat_shape_ok(d.vocab, h)) return fail(FL_ERR_ARG, "output.weight shape mismatch");
        if (T == 1) {
            int rc = keep_raw(m, &m->rout, type, d.vocab, h, raw, nbytes);
            if (rc) return rc;
            return upload_matrix(m, type, d.vocab, h, raw, nullptr, nullptr, &m->output, (double)nbytes);
        }
        std::vector<uint8_t> part = slice_rows(raw, type, h, rk * m->vocab_l, m->vocab_l);
        return upload_matrix(m, type, m->vocab_l, h, part.data(), nullptr, nullptr, &m->output, (double)part.size());
    }
    int l;
    std::string sfx;
    if (!parse_layer(name, &l, &sfx)) return FL_OK; /* tensors the forward pass does not read are ignored */
    if (l < 0 || l >= d.n_layers) return FL_OK;
    Layer& L = m->layers[(size_t)l];
    if (sfx == "attn_norm.weight") return upload_vector(m, type, raw, nbytes, h, &L.attn_norm);
    if (sfx == "ffn_norm.weight") return upload_vector(m, type, raw, nbytes, h, &L.ffn_norm);
    if (sfx == "post_attn_norm.weight") return upload_vector(m, type, raw, nbytes, h, &L.post_attn_norm);
    if (sfx == "post_ffn_norm.weight") return upload_vector(m, type, raw, nbytes, h, &L.post_ffn_norm);
    /* biases of this rank's heads (element slices of F32/F16 vectors) */
    auto bias = [&](int full, int local, float** out) -> int {
        if (T == 1) return upload_vector(m, type, raw, nbytes, full, out);
        if (block_elems(type) != 1) return fail(FL_ERR_UNSUPPORTED, "%s: quantized bias with tensor parallelism", name);
        const size_t eb = (size_t)block_bytes(type);
        return upload_vector(m, type, raw + (size_t)rk * local * eb, (uint64_t)local * eb, local, out);
    };
    if (sfx == "attn_q.bias") return bias(qd, m->qd_l, &L.bq);
    if (sfx == "attn_k.bias") return bias(kvd, m->kvd_l, &L.bk);
    if (sfx == "attn_v.bias") return bias(kvd, m->kvd_l, &L.bv);
    /* column-parallel (rows split: heads) and row-parallel (columns split) */
    struct { const char* s; DevMatrix* dm; int rows, cols, split_cols, lrows, lcols; } mats[] = {
        {"attn_q.weight", &L.wq, qd, h, 0, m->qd_l, h},
        {"attn_k.weight", &L.wk, kvd, h, 0, m->kvd_l, h},
        {"attn_v.weight", &L.wv, kvd, h, 0, m->kvd_l, h},
        {"attn_output.weight", &L.wo, h, qd, 1, h, m->qd_l},
        {"ffn_down.weight", &L.down, h, f, 1, h, m->ffn_l},
    };
    RawMatrix* raws[] = {&L.rq, &L.rk, &L.rv, &L.ro, &L.rdown};
    int mi = 0;
    for (auto& e : mats) {
        RawMatrix* rm = raws[mi++];
        if (sfx == e.s) {
            if (!mat_shape_ok(e.rows, e.cols)) return fail(FL_ERR_ARG, "%s shape mismatch", name);
            if (T == 1) {
                int rc = keep_raw(m, rm, type, e.rows, e.cols, raw, nbytes);
                if (rc) return rc;
                return upload_matrix(m, type, e.rows, e.cols, raw, nullptr, nullptr, e.dm, (double)nbytes);
            }
            if (e.split_cols && e.lcols % block_elems(type))
                return fail(FL_ERR_UNSUPPORTED, "%s: %d columns per rank are not whole blocks of type %d", name,
                            e.lcols, type);
            std::vector<uint8_t> part = e.split_cols ? slice_cols(raw, type, e.rows, e.cols, rk * e.lcols, e.lcols)
                                                     : slice_rows(raw, type, e.cols, rk * e.lrows, e.lrows);
            int rc = keep_raw(m, rm, type, e.lrows, e.lcols, part.data(), part.size()); /* this rank's slice */
            if (rc) return rc;
            return upload_matrix(m, type, e.lrows, e.lcols, part.data(), nullptr, nullptr, e.dm, (double)part.size());
        }
    }
    if (sfx == "ffn_gate.weight" || sfx == "ffn_up.weight") {
        if (!mat_shape_ok(f, h)) return fail(FL_ERR_ARG, "%s shape mismatch", name);
        if (f % 8) return fail(FL_ERR_UNSUPPORTED, "feed_forward_length %d is not a multiple of 8", f);
        const bool is_gate = sfx == "ffn_gate.weight";
        std::vector<uint8_t> part;
        if (T > 1) {
            part = slice_rows(raw, type, h, rk * m->ffn_l, m->ffn_l);
            raw = part.data();
            nbytes = part.size();
        }
        {
            int rc = keep_raw(m, is_gate ? &L.rgate : &L.rup, type, m->ffn_l, h, raw, nbytes);
            if (rc) return rc;
        }
        if (L.stash_type < 0) {
            L.stash.assign(raw, raw + nbytes);
            L.stash_type = type;
            L.stash_is_gate = is_gate;
            return FL_OK;
        }
        if (L.stash_is_gate == (int)is_gate) return fail(FL_ERR_ARG, "%s uploaded twice", name);
        if (L.stash_type != type)
            return fail(FL_ERR_UNSUPPORTED, "ffn_gate and ffn_up of layer %d have different types", l);
        const uint8_t* gate = is_gate ? raw : L.stash.data();
        const uint8_t* up = is_gate ? L.stash.data() : raw;
        /* interleave: tile t rows 0..7 = gate rows 8t.., rows 8..15 = up rows 8t.. */
        const int fl = m->ffn_l;
        std::vector<int32_t> map((size_t)2 * fl);
        for (int R = 0; R < 2 * fl; R++) {
            int t = R / 16, r = R % 16;
            map[(size_t)R] = r < 8 ? (8 * t + r) : (-1 - (8 * t + r - 8));
        }
        int rc = upload_matrix(m, type, 2 * fl, h, gate, up, map.data(), &L.gate_up, 2.0 * (double)nbytes);
        std::vector<uint8_t>().swap(L.stash);
        return rc;
    }
    return FL_OK;
}

extern "C" int fl_model_finalize(fl_model* m)
{
    if (!m) return fail(FL_ERR_ARG, "null model");
    if (m->group) {
        for (fl_model* r : m->ranks) {
            int rc = fl_model_finalize(r);
            if (rc) return rc;
        }
        m->finalized = true;
        return FL_OK;
    }
    if (m->finalized) return FL_OK;
    if (cudaSetDevice(m->d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    const fl_model_desc& d = m->d;
    if (!m->emb_raw) return fail(FL_ERR_STATE, "Required tensor 'token_embd.weight' not found in GGUF file.");
    if (!m->out_norm) return fail(FL_ERR_STATE, "Required tensor 'output_norm.weight' not found in GGUF file.");
    for (int l = 0; l < d.n_layers; l++) {
        Layer& L = m->layers[(size_t)l];
        const char* miss = nullptr;
        if (!L.attn_norm) miss = "attn_norm.weight";
        else if (!L.wq.present) miss = "attn_q.weight";
        else if (!L.wk.present) miss = "attn_k.weight";
        else if (!L.wv.present) miss = "attn_v.weight";
        else if (!L.wo.present) miss = "attn_output.weight";
        else if (!L.ffn_norm) miss = "ffn_norm.weight";
        else if (!L.gate_up.present) miss = L.stash_type >= 0 ? (L.stash_is_gate ? "ffn_up.weight" : "ffn_gate.weight")
                                                                : "ffn_gate.weight";
        else if (!L.down.present) miss = "ffn_down.weight";
        else if (d.arch == FL_ARCH_GEMMA2 && !L.post_attn_norm) miss = "post_attn_norm.weight";
        else if (d.arch == FL_ARCH_GEMMA2 && !L.post_ffn_norm) miss = "post_ffn_norm.weight";
        else if (d.arch == FL_ARCH_QWEN2 && (!L.bq || !L.bk || !L.bv)) miss = "attn_q/k/v.bias";
        if (miss) return fail(FL_ERR_STATE, "Required tensor 'blk.%d.%s' not found in GGUF file.", l, miss);
    }
    if (!m->output.present) {
        /* LoadTensorOptional("output.weight") ?? tokenEmbed (GgufModelLoader.cs:368-369) */
        if (m->T == 1) m->rout = RawMatrix{m->emb_raw, m->emb_type, d.vocab, d.hidden};
        std::vector<uint8_t> host((size_t)m->emb_bytes);
        CK(cudaMemcpy(host.data(), m->emb_raw, (size_t)m->emb_bytes, cudaMemcpyDeviceToHost));
        if (m->T > 1) host = slice_rows(host.data(), m->emb_type, d.hidden, m->rank * m->vocab_l, m->vocab_l);
        int rc = upload_matrix(m, m->emb_type, m->vocab_l, d.hidden, host.data(), nullptr, nullptr, &m->output,
                               (double)host.size());
        if (rc) return rc;
    }
    /* one embedding row per step */
    m->weight_bytes += (double)m->emb_bytes / d.vocab;
    m->finalized = true;
    return FL_OK;
}

extern "C" int fl_model_weight_bytes(fl_model* m, double* bytes)
{
    if (!m || !bytes) return fail(FL_ERR_ARG, "null argument");
    *bytes = m->weight_bytes;
    if (m->group) /* all ranks' shards */
        for (fl_model* r : m->ranks) *bytes += r->weight_bytes;
    return FL_OK;
}

/* ── session: the token step as a phase list for the persistent kernel ─── */
static void set_seg(FlMvArgs& a, int i, const DevMatrix& dm, const float* bias, int tile0)
{
    a.seg[i].w = dm.d;
    a.seg[i].bias = bias;
    a.seg[i].fmt = dm.L.fmt;
    a.seg[i].expanded = dm.L.expanded;
    a.seg[i].unit_bytes = dm.L.unit_bytes;
    a.seg[i].n_tiles = dm.L.n_tiles;
    a.seg[i].tile0 = tile0;
    a.seg[i].rows = dm.L.rows;
}

static FlMvArgs base_args(fl_session* s, const DevMatrix& dm, int K)
{
    FlMvArgs a;
    memset(&a, 0, sizeof a);
    set_seg(a, 0, dm, nullptr, 0);
    a.n_seg = 1;
    a.n_tiles = dm.L.n_tiles;
    a.n_kb = dm.L.n_kb;
    a.K = K;
    a.rows_total = dm.L.rows;
    a.err = s ? s->state + ST_ERR : nullptr;
    return a;
}

enum { CLS_MV = 0, CLS_ATTN = 1, CLS_OTHER = 2 };

static double mat_bytes(const DevMatrix& dm) { return (double)dm.L.gguf_bytes; }

struct PhaseList {
    std::vector<FlPhase> ph;
    std::vector<int> cls;
    std::vector<double> bytes;
    void add_mv(const FlMvArgs& a, double b)
    {
        FlPhase p;
        memset(&p, 0, sizeof p);
        p.kind = FL_PH_MATVEC;
        p.mv = a;
        ph.push_back(p);
        cls.push_back(CLS_MV);
        bytes.push_back(b);
    }
};

/* The ops of LlamaForwardPass.Forward (LlamaForwardPass.cs:82-130; Gemma2
 * post-norms Gemma2ForwardPass.cs:78-104; Qwen2 biases Qwen2ForwardPass.cs:
 * 83-85; Mistral window MistralForwardPass.cs:196) as phases. */
static void build_phases(fl_session* s, PhaseList& P)
{
    fl_model* m = s->m;
    const fl_model_desc& d = m->d;
    const int h = d.hidden, qd = m->qd_l, kvd = m->kvd_l, T = m->T;
    const bool gemma = d.arch == FL_ARCH_GEMMA2;
    int32_t* pos = s->state + ST_POS;
    /* Tensor parallelism, row exchanges: a row-parallel projection (Wo,
     * down) stores its partial rows as tagged 8-byte words into this rank's
     * receive slot [parity][rank] of every rank (tp_push), and the next
     * phase's prologue waits for the exchange's tags and sums the T slots of
     * its own region in rank order, with the residual or as Gemma's pending
     * post-norm input (tp_sum_in) — with no grid barrier in between.  The
     * residual stream alternates between xa and xb at every exchange.  (On one
     * GPU the projection adds into the residual in its epilogue and a grid
     * barrier separates the phases, which measured faster there.) */
    int xk = 0;
    auto slot_base = [&](uint8_t* region, int parity, int rank) {
        return reinterpret_cast<unsigned long long*>(region + FL_TP_RECV_OFF) +
               ((size_t)parity * FL_TP_MAX + rank) * s->xchg_recv_n;
    };
    auto tp_push = [&](FlMvArgs& a, int parity) {
        a.epi = FL_EPI_STORE;
        a.tp_n = T;
        a.push_x = xk + 1;
        for (int q = 0; q < T; q++) a.tp_out[q] = reinterpret_cast<float*>(slot_base(s->tp_peer[q], parity, m->rank));
    };
    auto tp_sum_in = [&](FlMvArgs& a, int parity) {
        a.tp_parts = T;
        a.part_stride = s->xchg_recv_n;
        a.parts = slot_base(s->xchg, parity, 0);
    };
    /* marks the phase just added as the one that reads exchange xk */
    auto after_exchange = [&]() { P.ph.back().xk = ++xk; };

    FlPhase e;
    memset(&e, 0, sizeof e);
    e.kind = FL_PH_EMBED;
    e.em.raw = m->emb_raw;
    e.em.ggml_type = m->emb_type;
    e.em.hidden = h;
    e.em.vocab = d.vocab;
    e.em.token = s->state + ST_TOKEN;
    e.em.x = s->xa;
    e.em.zero_buf = s->absmax;
    e.em.zero_n = s->n_absmax;
    e.em.err = s->state + ST_ERR;
    P.ph.push_back(e);
    P.cls.push_back(CLS_OTHER);
    P.bytes.push_back((double)m->emb_bytes / d.vocab);

    float* x = s->xa;
    float* x_other = s->xb;
    for (int l = 0; l < d.n_layers; l++) {
        Layer& L = m->layers[(size_t)l];
        float* amax_att = s->absmax + 2 * l;
        float* amax_act = s->absmax + 2 * l + 1;
        float* kc = s->kc + (size_t)l * s->max_ctx * kvd;
        float* vc = s->vc + (size_t)l * s->max_ctx * kvd;
        /* attention sub-layer: norm → q,k,v (+bias) → RoPE → KV append */
        FlMvArgs a = base_args(s, L.wq, h);
        set_seg(a, 0, L.wq, L.bq, 0);
        set_seg(a, 1, L.wk, L.bk, L.wq.L.n_tiles);
        set_seg(a, 2, L.wv, L.bv, L.wq.L.n_tiles + L.wk.L.n_tiles);
        a.n_seg = 3;
        a.n_tiles = L.wq.L.n_tiles + L.wk.L.n_tiles + L.wv.L.n_tiles;
        const bool x_after_down = T > 1 && l > 0; /* x + the ranks' down rows */
        if (!gemma) {
            a.in_mode = FL_IN_RMSNORM;
            a.x = x;
            a.norm_w = L.attn_norm;
            a.eps = d.rms_eps;
            if (x_after_down) {
                tp_sum_in(a, 1);
                a.resid_out = x_other;
                std::swap(x, x_other);
            }
        } else if (l == 0) {
            a.in_mode = FL_IN_GEMMA_NORM;
            a.x = x;
            a.norm_w = L.attn_norm;
            a.eps = 1e-6f;
        } else {
            a.in_mode = FL_IN_GEMMA_RESID;
            a.x = x;
            a.pend = s->o;
            a.pend_w = m->layers[(size_t)l - 1].post_ffn_norm;
            a.resid_out = x_other;
            a.norm_w = L.attn_norm;
            a.eps = 1e-6f;
            if (x_after_down) tp_sum_in(a, 1);
            std::swap(x, x_other);
        }
        a.epi = FL_EPI_QKV;
        a.q_rows = qd;
        a.kv_rows = kvd;
        a.head_dim = d.head_dim;
        a.rope_cs = m->rope_cs;
        a.pos = pos;
        a.q_out = s->q;
        a.k_cache = kc;
        a.v_cache = vc;
        P.add_mv(a, mat_bytes(L.wq) + mat_bytes(L.wk) + mat_bytes(L.wv) + 4.0 * h);
        if (x_after_down) after_exchange();

        FlPhase at;
        memset(&at, 0, sizeof at);
        at.kind = FL_PH_ATTN;
        at.at.q = s->q;
        at.at.k_cache = kc;
        at.at.v_cache = vc;
        at.at.out = s->att;
        at.at.out_absmax = amax_att;
        at.at.part = s->attn_part;
        at.at.counter = s->attn_counter;
        at.at.pos = pos;
        at.at.n_heads = m->nh_l;
        at.at.n_kv = m->nkv_l;
        at.at.head_dim = d.head_dim;
        at.at.n_split = s->attn_split;
        int window = INT_MAX;
        if (d.arch == FL_ARCH_MISTRAL) window = d.sliding_window;
        if (gemma && (l % 2) == 0) window = d.sliding_window; /* Gemma2ForwardPass.cs:87 */
        at.at.window = window > 0 ? window : INT_MAX;
        at.at.scale = d.attn_scale;
        at.at.softcap = gemma ? d.attn_softcap : 0.0f;
        at.at.err = s->state + ST_ERR;
        P.ph.push_back(at);
        P.cls.push_back(CLS_ATTN);
        P.bytes.push_back(0.0);
        at.kind = FL_PH_ATTN_COMBINE;
        P.ph.push_back(at);
        P.cls.push_back(CLS_ATTN);
        P.bytes.push_back(0.0);

        /* output projection + residual (Gemma: post-attention norm first) */
        a = base_args(s, L.wo, qd);
        a.in_mode = FL_IN_PLAIN;
        a.x = s->att;
        a.absmax = amax_att;
        a.epi = gemma ? FL_EPI_STORE : FL_EPI_RESID;
        a.y = gemma ? s->o : x;
        if (T > 1) tp_push(a, 0);
        P.add_mv(a, mat_bytes(L.wo));

        /* FFN: norm → gate/up → SiLU|GELU(gate)*up */
        a = base_args(s, L.gate_up, h);
        if (!gemma) {
            a.in_mode = FL_IN_RMSNORM;
            a.x = x;
            a.norm_w = L.ffn_norm;
            a.eps = d.rms_eps;
            if (T > 1) {
                tp_sum_in(a, 0);
                a.resid_out = x_other;
                std::swap(x, x_other);
            }
        } else {
            a.in_mode = FL_IN_GEMMA_RESID;
            a.x = x;
            a.pend = s->o;
            a.pend_w = L.post_attn_norm;
            a.resid_out = x_other;
            a.norm_w = L.ffn_norm;
            a.eps = 1e-6f;
            if (T > 1) tp_sum_in(a, 0);
            std::swap(x, x_other);
        }
        a.epi = FL_EPI_GLU;
        a.rows_total = m->ffn_l;
        a.act_gelu = gemma ? 1 : 0;
        a.act_out = s->act;
        a.act_absmax = amax_act;
        P.add_mv(a, mat_bytes(L.gate_up) + 4.0 * h);
        if (T > 1) after_exchange();

        a = base_args(s, L.down, m->ffn_l);
        a.in_mode = FL_IN_PLAIN;
        a.x = s->act;
        a.absmax = amax_act;
        a.epi = gemma ? FL_EPI_STORE : FL_EPI_RESID;
        a.y = gemma ? s->o : x;
        if (T > 1) tp_push(a, 1);
        P.add_mv(a, mat_bytes(L.down));
    }
    /* final norm + LM head + greedy argmax */
    FlMvArgs a = base_args(s, m->output, h);
    if (!gemma) {
        a.in_mode = FL_IN_RMSNORM;
        a.x = x;
        a.norm_w = m->out_norm;
        a.eps = d.rms_eps;
        if (T > 1) {
            tp_sum_in(a, 1);
            a.resid_out = x_other;
        }
    } else {
        a.in_mode = FL_IN_GEMMA_RESID;
        a.x = x;
        a.pend = s->o;
        a.pend_w = m->layers.back().post_ffn_norm;
        a.resid_out = x_other;
        a.norm_w = m->out_norm;
        a.eps = 1e-6f;
        if (T > 1) tp_sum_in(a, 1);
    }
    a.epi = FL_EPI_LOGITS;
    a.y = s->logits;
    a.softcap = gemma ? d.final_softcap : 0.0f;
    if (T > 1) {
        /* vocabulary-parallel head: logits rows [rank*V/T, ...) to every rank */
        a.tp_n = T;
        a.tp_row0 = m->rank * m->vocab_l;
        for (int q = 0; q < T; q++) a.tp_out[q] = reinterpret_cast<float*>(s->tp_peer[q] + s->xchg_logits_off);
    }
    a.cta_best = s->cta_best;
    a.counter = s->state + ST_HEADCNT;
    a.argmax_out = s->state + ST_ARGMAX;
    P.add_mv(a, mat_bytes(m->output) + 4.0 * h);
    if (T > 1) after_exchange();
    s->tp_rows_per_step = xk;
}

/* One token step: zero the grid-barrier counter, then the persistent kernel. */
static int enqueue_step(fl_session* s)
{
    CK(cudaMemsetAsync(s->bar, 0, 4, s->st));
    CK(fl_launch_token(s->tk_kernel, s->ta, s->tk_grid, s->tk_smem, s->st));
    return FL_OK;
}

static int session_build(fl_session* s);

extern "C" int fl_session_create(fl_model* m, int32_t max_ctx, int32_t max_batch, int32_t kv_dtype, fl_session** out)
{
    if (!m || !out) return fail(FL_ERR_ARG, "null argument");
    if (!m->finalized) {
        int rc = fl_model_finalize(m);
        if (rc) return rc;
    }
    if (m->group) return group_session_create(m, max_ctx, max_batch, kv_dtype, out);
    if (kv_dtype != FL_KV_F32) return fail(FL_ERR_UNSUPPORTED, "kv dtype %d", kv_dtype);
    if (max_batch < 1) max_batch = 1;
    if (max_batch > 1 && m->T > 1) return fail(FL_ERR_UNSUPPORTED, "batched sessions run on one GPU (tp_size 1)");
    const fl_model_desc& d = m->d;
    if (max_ctx <= 0 || max_ctx > d.max_ctx) max_ctx = d.max_ctx;
    if (cudaSetDevice(d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    const void* tk_kernel = fl_token_kernel_ptr(d.head_dim, d.n_heads / d.n_kv_heads);
    if (!tk_kernel)
        return fail(FL_ERR_UNSUPPORTED, "no token kernel for head_dim %d with %d query heads per kv head", d.head_dim,
                    d.n_heads / d.n_kv_heads);
    int max_dyn = 0;
    if (fl_token_configure(tk_kernel, &max_dyn) != cudaSuccess) return fail(FL_ERR_CUDA, "token kernel configuration failed");
    fl_session* s = new fl_session();
    s->m = m;
    s->max_ctx = max_ctx;
    s->max_dyn = max_dyn;
    s->tk_kernel = tk_kernel;
    /* this rank's share of the model (the whole model without tensor parallelism) */
    const int h = d.hidden, qd = m->qd_l, kvd = m->kvd_l, grp = d.n_heads / d.n_kv_heads;
    const int G = m->sm_count;
    /* attention items (kv head, split): at most one per SM, and at most 32
     * splits per kv head, so that the split merge reads each split's (max,
     * sum) in one warp load (a tensor-parallel rank keeps few kv heads) */
    int split = G / m->nkv_l;
    if (split > 32) split = 32;
    if (split > max_ctx) split = max_ctx;
    if (split < 1) split = 1;
    s->attn_split = split;
    s->n_absmax = 2 * d.n_layers;
    int rc = FL_OK;
    s->n_slots = max_batch;
    s->slot_stride = (size_t)d.n_layers * max_ctx * kvd;
    s->slot_len.assign((size_t)max_batch, 0);
    size_t kv_bytes = (size_t)max_batch * d.n_layers * max_ctx * kvd * 4;
#define AL(p, b) if (!rc) rc = dalloc(s->allocs, &(p), (b))
    AL(s->xa, (size_t)h * 4);
    AL(s->xb, (size_t)h * 4);
    AL(s->o, (size_t)h * 4);
    AL(s->q, (size_t)qd * 4);
    AL(s->att, (size_t)qd * 4);
    AL(s->act, (size_t)m->ffn_l * 4);
    /* receive words of the row exchanges: 8 bytes per row (value, tag) */
    s->xchg_recv_n = (h + 63) & ~63;
    if (m->T == 1) {
        AL(s->logits, (size_t)d.vocab * 4);
    } else {
        /* the exchange region peers write into; the full logits live at its end */
        s->xchg_logits_off = FL_TP_RECV_OFF + (size_t)2 * FL_TP_MAX * s->xchg_recv_n * 8;
        /* then the prompt path's partial sums: two slots of pf_tp_rows x hidden floats */
        s->pf_tp_rows = std::min(max_ctx, 2048);
        s->xchg_pf_off = (s->xchg_logits_off + (size_t)d.vocab * 4 + 255) & ~(size_t)255;
        s->xchg_bytes = s->xchg_pf_off + (size_t)2 * s->pf_tp_rows * h * 4;
        AL(s->xchg, s->xchg_bytes);
        AL(s->tp_epoch, 16);
        if (!rc) s->logits = reinterpret_cast<float*>(s->xchg + s->xchg_logits_off);
    }
    AL(s->kc, kv_bytes);
    AL(s->vc, kv_bytes);
    AL(s->absmax, (size_t)s->n_absmax * 4);
    AL(s->state, (size_t)ST_N * 4);
    AL(s->attn_counter, (size_t)m->nkv_l * 4);
    AL(s->attn_part, (size_t)m->nkv_l * split * grp * (d.head_dim + 2) * 4);
    AL(s->cta_best, (size_t)G * 8 + 8);
    AL(s->out_tokens, (size_t)max_ctx * 4 + 4);
    s->topk_scratch_bytes = fl_topk_scratch_bytes(d.vocab, 0);
    AL(s->topk_scratch, s->topk_scratch_bytes);
    AL(s->topk_ids, (size_t)d.vocab * 4);
    AL(s->topk_vals, (size_t)d.vocab * 4);
    AL(s->bar, 16);
#undef AL
    if (rc) {
        fl_session_destroy(s);
        return rc;
    }
    if (cudaMallocHost(&s->h_state, ST_N * 4) != cudaSuccess ||
        cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking) != cudaSuccess) {
        fl_session_destroy(s);
        return fail(FL_ERR_CUDA, "stream/pinned allocation failed");
    }
    cudaMemsetAsync(s->state, 0, ST_N * 4, s->st);
    cudaMemsetAsync(s->attn_counter, 0, (size_t)m->nkv_l * 4, s->st);
    cudaMemsetAsync(s->kc, 0, kv_bytes, s->st);
    cudaMemsetAsync(s->vc, 0, kv_bytes, s->st);
    if (s->xchg) {
        cudaMemsetAsync(s->xchg, 0, s->xchg_bytes, s->st);
        cudaMemsetAsync(s->tp_epoch, 0, 16, s->st);
    }
    if (cudaStreamSynchronize(s->st) != cudaSuccess) {
        fl_session_destroy(s);
        return fail(FL_ERR_CUDA, "session init failed");
    }
    if (m->T > 1) { /* built by fl_session_tp_connect once the peers are mapped */
        *out = s;
        return FL_OK;
    }
    rc = session_build(s);
    if (rc) {
        fl_session_destroy(s);
        return rc;
    }
    *out = s;
    return FL_OK;
}

/* The phase list, the persistent kernel's configuration and the captured
 * token graph (after the peers are mapped, with tensor parallelism). */
static int session_build(fl_session* s)
{
    fl_model* m = s->m;
    const fl_model_desc& d = m->d;
    const int G = m->sm_count, grp = d.n_heads / d.n_kv_heads, max_ctx = s->max_ctx, max_dyn = s->max_dyn;
    int rc = FL_OK;
    /* phase list */
    PhaseList P;
    build_phases(s, P);
    s->n_phases = (int)P.ph.size();
    s->phase_cls = P.cls;
    s->phase_bytes = P.bytes;
    std::vector<FlFeedPhase> feed;
    for (const FlPhase& p : P.ph)
        if (p.kind == FL_PH_MATVEC) {
            FlFeedPhase f;
            memset(&f, 0, sizeof f);
            f.n_kb = p.mv.n_kb;
            f.n_tiles = p.mv.n_tiles;
            f.n_seg = p.mv.n_seg;
            for (int i = 0; i < p.mv.n_seg; i++) {
                f.tile0[i] = p.mv.seg[i].tile0;
                f.unit_bytes[i] = p.mv.seg[i].unit_bytes;
                f.w[i] = p.mv.seg[i].w;
            }
            feed.push_back(f);
        }
    rc = dalloc(s->allocs, &s->d_phases, P.ph.size() * sizeof(FlPhase));
    if (!rc) rc = dalloc(s->allocs, &s->d_feed, feed.size() * sizeof(FlFeedPhase));
    if (!rc) rc = dalloc(s->allocs, &s->timestamps, (P.ph.size() + 1) * 8);
    if (!rc) rc = dalloc(s->allocs, &s->cta_done, P.ph.size() * (size_t)G * 8);
    if (!rc) rc = dalloc(s->allocs, &s->detail, P.ph.size() * (size_t)(FL_TK_WARPS * 4 + 1) * 8);
    if (rc) return rc;
    /* shared memory: weight ring of the largest unit + x-encoding / attention scratch */
    int slot = 0, max_kb = 0, max_tiles = 0;
    for (const FlPhase& p : P.ph)
        if (p.kind == FL_PH_MATVEC) {
            for (int i = 0; i < p.mv.n_seg; i++) slot = std::max(slot, p.mv.seg[i].unit_bytes);
            max_kb = std::max(max_kb, p.mv.n_kb);
            max_tiles = std::max(max_tiles, (p.mv.n_tiles + G - 1) / G);
        }
    if (max_tiles > FL_TK_MAX_TILES)
        return fail(FL_ERR_UNSUPPORTED, "a projection has %d row tiles per SM (limit %d)", max_tiles, FL_TK_MAX_TILES);
    slot = (slot + 127) & ~127;
    const size_t xenc = (size_t)max_kb * 8 * FL_XENC_CHUNK_BYTES;
    /* attention: q, per-warp outputs, reductions, the scores of one item */
    const int span = d.sliding_window > 0 ? std::min(max_ctx, d.sliding_window) : max_ctx;
    const int per_max = (span + s->attn_split - 1) / s->attn_split;
    const size_t attn =
        (size_t)(grp * d.head_dim + FL_TK_WARPS * grp * d.head_dim + FL_TK_WARPS * 8 * 2 + per_max * grp) * 4;
    size_t scratch = std::max(xenc, attn);
    if (m->T > 1) {
        /* a phase after a row exchange (Wo, down) stages x + the ranks' rows
         * (hidden floats) at the end of the scratch, behind the encoding, and
         * its prologue keeps the input in registers (<= 64 k-blocks) */
        if (d.hidden % 4 || d.hidden > 64 * 256)
            return fail(FL_ERR_UNSUPPORTED, "tensor parallelism needs hidden a multiple of 4, at most 16384 (%d)",
                        d.hidden);
        const size_t enc_h = (size_t)((d.hidden + 255) / 256) * 8 * FL_XENC_CHUNK_BYTES;
        scratch = std::max(scratch, ((enc_h + 15) & ~(size_t)15) + (size_t)d.hidden * 4);
    }
    scratch = (scratch + 15) & ~(size_t)15;
    const int n_feed = (int)feed.size();
    int n_slots = 1;
    while (n_slots < FL_TK_MAX_SLOTS && fl_token_smem_bytes(n_slots + 1, slot, scratch, n_feed) <= (size_t)max_dyn)
        n_slots++;
    if (fl_token_smem_bytes(n_slots, slot, scratch, n_feed) > (size_t)max_dyn)
        return fail(FL_ERR_UNSUPPORTED, "shared memory budget exceeded (x encoding %zu B, %d stream descriptors)", xenc,
                    n_feed);
    FlTokenArgs& ta = s->ta;
    memset(&ta, 0, sizeof ta);
    ta.phases = s->d_phases;
    ta.feed = s->d_feed;
    ta.n_feed = (int)feed.size();
    ta.n_phases = s->n_phases;
    ta.n_slots = n_slots;
    ta.slot_bytes = slot;
    ta.scratch_bytes = scratch;
    ta.bar = s->bar;
    ta.err = s->state + ST_ERR;
    ta.timestamps = s->timestamps;
    ta.cta_done = s->cta_done;
    ta.detail = s->detail;
    ta.advance = 1;
    ta.token = s->state + ST_TOKEN;
    ta.pos = s->state + ST_POS;
    ta.out_tokens = s->out_tokens;
    ta.step = s->state + ST_STEP;
    ta.tp_epoch = s->tp_epoch;
    ta.tp_rows_per_step = s->tp_rows_per_step;
    if (m->T > 1) {
        ta.tp_size = m->T;
        ta.tp_rank = m->rank;
        ta.tp_n_exchanges = 1;
        ta.tp_recv_n = s->xchg_recv_n;
        ta.tp_epoch = s->tp_epoch;
        for (int q = 0; q < m->T; q++) ta.tp_peer[q] = s->tp_peer[q];
    }
    s->tk_smem = fl_token_smem_bytes(n_slots, slot, scratch, n_feed);
    s->tk_grid = G;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, s->tk_kernel, 32 * FL_TK_WARPS, s->tk_smem) !=
            cudaSuccess ||
        per_sm < 1)
        return fail(FL_ERR_UNSUPPORTED, "the token kernel does not fit one CTA per SM");
    CK(cudaMemcpyAsync(s->d_phases, P.ph.data(), P.ph.size() * sizeof(FlPhase), cudaMemcpyHostToDevice, s->st));
    CK(cudaMemcpyAsync(s->d_feed, feed.data(), feed.size() * sizeof(FlFeedPhase), cudaMemcpyHostToDevice, s->st));
    CK(cudaStreamSynchronize(s->st));
    /* capture the token step once */
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
    rc = enqueue_step(s);
    cudaError_t ce = cudaStreamEndCapture(s->st, &g);
    if (rc || ce != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return rc ? rc : fail(FL_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ce));
    }
    ce = cudaGraphInstantiate(&s->graph, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return fail(FL_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ce));
    s->launches = 1;
    s->built = true;
    return FL_OK;
}

static void forget_regions(const fl_session* s);

extern "C" void fl_session_destroy(fl_session* s)
{
    if (!s) return;
    if (s->group) return group_session_destroy(s);
    forget_regions(s);
    cudaSetDevice(s->m->d.device);
    if (s->st) cudaStreamSynchronize(s->st);
    if (s->graph) cudaGraphExecDestroy(s->graph);
    for (void* p : s->tp_opened)
        if (p) cudaIpcCloseMemHandle(p);
    for (void* p : s->allocs) cudaFree(p);
    if (s->h_state) cudaFreeHost(s->h_state);
    if (s->st) cudaStreamDestroy(s->st);
    delete s;
}

/* ── tensor parallelism: mapping the ranks' exchange regions ────────────── */

/* Exchange regions handed out by this process: a rank whose peers live in
 * the same process (one host thread per GPU) maps them directly with peer
 * access, since CUDA IPC does not open a process's own handles. */
struct LocalRegion {
    uint8_t handle[FL_TP_HANDLE_BYTES];
    int device;
    uint8_t* ptr;
    const fl_session* owner;
};
static std::mutex g_regions_mu;
static std::vector<LocalRegion> g_regions;

static void forget_regions(const fl_session* s)
{
    std::lock_guard<std::mutex> lk(g_regions_mu);
    g_regions.erase(std::remove_if(g_regions.begin(), g_regions.end(),
                                   [s](const LocalRegion& r) { return r.owner == s; }),
                    g_regions.end());
}

extern "C" int fl_session_tp_handle(fl_session* s, void* handle)
{
    if (!s || !handle) return fail(FL_ERR_ARG, "null argument");
    if (s->group) return fail(FL_ERR_STATE, "a group session connects its ranks itself");
    if (s->m->T == 1) return fail(FL_ERR_STATE, "the model is not tensor-parallel");
    if (cudaSetDevice(s->m->d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, s->xchg));
    static_assert(sizeof(cudaIpcMemHandle_t) == FL_TP_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof h);
    LocalRegion r;
    memcpy(r.handle, &h, sizeof h);
    r.device = s->m->d.device;
    r.ptr = s->xchg;
    r.owner = s;
    std::lock_guard<std::mutex> lk(g_regions_mu);
    for (const LocalRegion& e : g_regions)
        if (e.owner == s) return FL_OK;
    g_regions.push_back(r);
    return FL_OK;
}

extern "C" int fl_session_tp_connect(fl_session* s, const void* handles)
{
    if (!s || !handles) return fail(FL_ERR_ARG, "null argument");
    if (s->group) return fail(FL_ERR_STATE, "a group session connects its ranks itself");
    fl_model* m = s->m;
    if (m->T == 1) return fail(FL_ERR_STATE, "the model is not tensor-parallel");
    if (s->built) return fail(FL_ERR_STATE, "the session is already connected");
    if (cudaSetDevice(m->d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    for (int q = 0; q < m->T; q++) {
        if (q == m->rank) {
            s->tp_peer[q] = s->xchg;
            continue;
        }
        const uint8_t* hq = static_cast<const uint8_t*>(handles) + (size_t)q * FL_TP_HANDLE_BYTES;
        LocalRegion local = {};
        bool is_local = false;
        {
            std::lock_guard<std::mutex> lk(g_regions_mu);
            for (const LocalRegion& e : g_regions)
                if (!memcmp(e.handle, hq, FL_TP_HANDLE_BYTES)) {
                    local = e;
                    is_local = true;
                    break;
                }
        }
        if (is_local) { /* a peer in this process: its pointer, with peer access */
            /* The ranks' kernels wait on one another, so each needs a GPU of
             * its own: two on one device are not guaranteed to be resident
             * together.  (A mapping from another process does not tell its
             * owner's device, so that case rests on the caller.) */
            if (local.device == m->d.device) return fail(FL_ERR_ARG, "ranks %d and %d share device %d", m->rank, q, local.device);
            cudaError_t pe = cudaDeviceEnablePeerAccess(local.device, 0);
            if (pe == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else if (pe != cudaSuccess)
                return fail(FL_ERR_CUDA, "peer access to device %d: %s", local.device, cudaGetErrorString(pe));
            s->tp_peer[q] = local.ptr;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hq, sizeof h);
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return fail(FL_ERR_CUDA, "mapping rank %d's exchange region: %s", q, cudaGetErrorString(e));
        s->tp_opened[q] = p;
        s->tp_peer[q] = static_cast<uint8_t*>(p);
    }
    return session_build(s);
}

extern "C" int fl_session_reset(fl_session* s, int32_t seq_slot)
{
    if (!s) return fail(FL_ERR_ARG, "null session");
    if (s->group) {
        for (fl_session* r : s->ranks) {
            int rc = fl_session_reset(r, seq_slot);
            if (rc) return rc;
        }
        return FL_OK;
    }
    if (seq_slot < 0 || seq_slot >= s->n_slots)
        return fail(FL_ERR_ARG, "sequence slot %d outside [0, %d)", seq_slot, s->n_slots);
    if (seq_slot == 0) s->cur_len = 0;
    else s->slot_len[(size_t)seq_slot] = 0;
    return FL_OK;
}

extern "C" int fl_session_tp_reset(fl_session* s)
{
    if (!s) return fail(FL_ERR_ARG, "null session");
    if (s->group) {
        for (fl_session* r : s->ranks) {
            int rc = fl_session_tp_reset(r);
            if (rc) return rc;
        }
        return FL_OK;
    }
    if (s->m->T == 1 || !s->xchg || !s->tp_epoch) return fail(FL_ERR_STATE, "not a tensor-parallel session");
    /* this rank's counters, the flags its peers raise in its region and the
     * receive words (their tags restart with the counters, so no word of an
     * earlier exchange may survive) */
    CK(cudaMemsetAsync(s->tp_epoch, 0, 16, s->st));
    CK(cudaMemsetAsync(s->xchg + FL_TP_FLAGS_OFF, 0,
                       FL_TP_RECV_OFF - FL_TP_FLAGS_OFF + (size_t)2 * FL_TP_MAX * s->xchg_recv_n * 8, s->st));
    CK(cudaStreamSynchronize(s->st));
    s->pf_epoch = 0;
    s->cur_len = 0;
    return FL_OK;
}

extern "C" int fl_session_launches_per_step(fl_session* s, int32_t* n)
{
    if (!s || !n) return fail(FL_ERR_ARG, "null argument");
    if (s->group) return fl_session_launches_per_step(s->ranks[0], n);
    *n = s->launches;
    return FL_OK;
}

static int check_device_err(fl_session* s)
{
    int32_t err = 0;
    CK(cudaMemcpy(&err, s->state + ST_ERR, 4, cudaMemcpyDeviceToHost));
    if (err == 0) return FL_OK;
    int32_t zero = 0;
    cudaMemcpy(s->state + ST_ERR, &zero, 4, cudaMemcpyHostToDevice);
    if (err == 1) return fail(FL_ERR_TIMEOUT, "a bounded device wait expired");
    if (err == 3)
        return fail(FL_ERR_UNSUPPORTED,
                    "a value of the prompt path or batched step is outside the fp16 range of its tensor-core operands "
                    "(|weight| > 255.9 or |activation| > 65504): feed these tokens through fl_forward");
    return fail(FL_ERR_ARG, "device reported error %d", err);
}

static int set_state(fl_session* s, int token, int pos)
{
    s->h_state[ST_TOKEN] = token;
    s->h_state[ST_POS] = pos;
    s->h_state[ST_ARGMAX] = 0;
    s->h_state[ST_STEP] = 0;
    CK(cudaMemcpyAsync(s->state, s->h_state, 4 * 4, cudaMemcpyHostToDevice, s->st));
    return FL_OK;
}

/* The checks of one token step (LlamaForwardPass.cs:85-93, KvCache.Append). A
 * group runs them on rank 0 before any rank launches: the ranks' states are
 * identical, and a rank that refused while the others launched would leave
 * them waiting for its exchanges. */
static int check_forward(const fl_session* s, int32_t token, int32_t position)
{
    if (!s->built) return fail(FL_ERR_STATE, "tensor-parallel session not connected (fl_session_tp_connect)");
    const fl_model_desc& d = s->m->d;
    if ((uint32_t)token >= (uint32_t)d.vocab)
        return fail(FL_ERR_ARG, "Token id %d is outside the valid vocabulary range [0, %d].", token, d.vocab - 1);
    if (position < 0 || position >= s->max_ctx)
        return fail(FL_ERR_ARG, "position %d is outside the KV cache [0, %d)", position, s->max_ctx);
    if (position > s->cur_len)
        return fail(FL_ERR_ARG, "position %d skips cached positions (cache holds %d)", position, s->cur_len);
    return FL_OK;
}

extern "C" int fl_forward(fl_session* s, int32_t token, int32_t position, float* logits, int32_t* argmax)
{
    if (!s) return fail(FL_ERR_ARG, "null session");
    if (s->group) {
        int rc = check_forward(s->ranks[0], token, position);
        if (rc) return rc;
        return run_ranks(s, [&](int r) {
            return fl_forward(s->ranks[r], token, position, r ? nullptr : logits, r ? nullptr : argmax);
        });
    }
    int rc = check_forward(s, token, position);
    if (rc) return rc;
    const fl_model_desc& d = s->m->d;
    if (cudaSetDevice(d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    rc = set_state(s, token, position);
    if (rc) return rc;
    CK(cudaGraphLaunch(s->graph, s->st));
    if (logits) CK(cudaMemcpyAsync(logits, s->logits, (size_t)d.vocab * 4, cudaMemcpyDeviceToHost, s->st));
    if (argmax) CK(cudaMemcpyAsync(&s->h_state[ST_ARGMAX], s->state + ST_ARGMAX, 4, cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
    rc = check_device_err(s);
    if (rc) return rc;
    if (argmax) *argmax = s->h_state[ST_ARGMAX];
    s->cur_len = position + 1;
    return FL_OK;
}

static int check_steps(const fl_session* s, int32_t token, int32_t start_pos, int32_t n_steps)
{
    if (!s->built) return fail(FL_ERR_STATE, "tensor-parallel session not connected (fl_session_tp_connect)");
    const fl_model_desc& d = s->m->d;
    if ((uint32_t)token >= (uint32_t)d.vocab) return fail(FL_ERR_ARG, "Token id %d is outside the vocabulary", token);
    if (start_pos < 0 || start_pos > s->cur_len || n_steps < 0 || start_pos + n_steps > s->max_ctx)
        return fail(FL_ERR_ARG, "steps [%d, %d) do not fit the KV cache (holds %d of %d)", start_pos,
                    start_pos + n_steps, s->cur_len, s->max_ctx);
    return FL_OK;
}

static int run_steps(fl_session* s, int32_t token, int32_t start_pos, int32_t n_steps, float* ms)
{
    int rc = check_steps(s, token, start_pos, n_steps);
    if (rc) return rc;
    const fl_model_desc& d = s->m->d;
    if (cudaSetDevice(d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    rc = set_state(s, token, start_pos);
    if (rc) return rc;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ms) {
        CK(cudaEventCreate(&e0));
        CK(cudaEventCreate(&e1));
        CK(cudaEventRecord(e0, s->st));
    }
    for (int i = 0; i < n_steps; i++) CK(cudaGraphLaunch(s->graph, s->st));
    if (ms) CK(cudaEventRecord(e1, s->st));
    CK(cudaStreamSynchronize(s->st));
    if (ms) {
        cudaEventElapsedTime(ms, e0, e1);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    rc = check_device_err(s);
    if (rc) return rc;
    s->cur_len = start_pos + n_steps;
    return FL_OK;
}

extern "C" int fl_decode_greedy(fl_session* s, int32_t token, int32_t start_pos, int32_t n_steps, int32_t* out_tokens)
{
    if (!s) return fail(FL_ERR_ARG, "null session");
    if (s->group) {
        int rc = check_steps(s->ranks[0], token, start_pos, n_steps);
        if (rc) return rc;
        return run_ranks(s, [&](int r) {
            return fl_decode_greedy(s->ranks[r], token, start_pos, n_steps, r ? nullptr : out_tokens);
        });
    }
    int rc = run_steps(s, token, start_pos, n_steps, nullptr);
    if (rc) return rc;
    if (out_tokens && n_steps > 0) CK(cudaMemcpy(out_tokens, s->out_tokens, (size_t)n_steps * 4, cudaMemcpyDeviceToHost));
    return FL_OK;
}

extern "C" int fl_time_decode(fl_session* s, int32_t token, int32_t start_pos, int32_t n_steps, float* ms)
{
    if (!s || !ms) return fail(FL_ERR_ARG, "null argument");
    if (s->group) { /* the slowest rank's time */
        int rc = check_steps(s->ranks[0], token, start_pos, n_steps);
        if (rc) return rc;
        std::vector<float> t(s->ranks.size(), 0.0f);
        rc = run_ranks(s, [&](int r) { return fl_time_decode(s->ranks[r], token, start_pos, n_steps, &t[(size_t)r]); });
        if (rc) return rc;
        *ms = *std::max_element(t.begin(), t.end());
        return FL_OK;
    }
    return run_steps(s, token, start_pos, n_steps, ms);
}

/* One step, with the phase boundaries read from the globaltimer stamps the
 * kernel records (CTA 0, after each grid barrier). */
extern "C" int fl_profile_step(fl_session* s, int32_t token, int32_t position, double* ms, double* bytes,
                               int32_t* launches)
{
    if (s && s->group) return fail(FL_ERR_UNSUPPORTED, "measurement hook of one rank: not available on a group session");
    if (s && !s->built) return fail(FL_ERR_STATE, "tensor-parallel session not connected (fl_session_tp_connect)");
    if (!s || !ms || !bytes) return fail(FL_ERR_ARG, "null argument");
    const fl_model_desc& d = s->m->d;
    if ((uint32_t)token >= (uint32_t)d.vocab || position < 0 || position >= s->max_ctx || position > s->cur_len)
        return fail(FL_ERR_ARG, "bad token/position");
    if (cudaSetDevice(d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    int rc = set_state(s, token, position);
    if (rc) return rc;
    CK(cudaGraphLaunch(s->graph, s->st));
    CK(cudaStreamSynchronize(s->st));
    rc = check_device_err(s);
    if (rc) return rc;
    std::vector<uint64_t> ts((size_t)s->n_phases + 1);
    CK(cudaMemcpy(ts.data(), s->timestamps, ts.size() * 8, cudaMemcpyDeviceToHost));
    for (int i = 0; i < FL_PROF_N; i++) {
        ms[i] = 0;
        bytes[i] = 0;
    }
    for (int p = 0; p < s->n_phases; p++) {
        const double t = (double)(ts[(size_t)p + 1] - ts[(size_t)p]) * 1e-6;
        ms[s->phase_cls[(size_t)p]] += t;
        bytes[s->phase_cls[(size_t)p]] += s->phase_bytes[(size_t)p];
        ms[FL_PROF_STEP] += t;
        bytes[FL_PROF_STEP] += s->phase_bytes[(size_t)p];
    }
    if (launches) *launches = s->launches;
    s->cur_len = position + 1;
    return FL_OK;
}

extern "C" int fl_topk(fl_session* s, int32_t k, int32_t* ids, float* vals, float* threshold)
{
    if (!s || !ids || !vals) return fail(FL_ERR_ARG, "null argument");
    if (s->group) return fl_topk(s->ranks[0], k, ids, vals, threshold); /* every rank holds the full logits */
    if (!s->built) return fail(FL_ERR_STATE, "tensor-parallel session not connected (fl_session_tp_connect)");
    const fl_model_desc& d = s->m->d;
    if (k < 1 || k > d.vocab) return fail(FL_ERR_ARG, "k must be in [1, %d]", d.vocab);
    if (cudaSetDevice(d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    CK(fl_launch_topk(s->logits, d.vocab, k, s->topk_ids, s->topk_vals, s->topk_scratch, s->topk_scratch_bytes, s->st));
    CK(cudaMemcpyAsync(ids, s->topk_ids, (size_t)k * 4, cudaMemcpyDeviceToHost, s->st));
    CK(cudaMemcpyAsync(vals, s->topk_vals, (size_t)k * 4, cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
    if (threshold) *threshold = vals[k - 1];
    return FL_OK;
}

extern "C" int fl_sample(fl_session* s, const fl_sampler_desc* sd, const int32_t* generated, int32_t n_generated,
                         float u, int32_t* token)
{
    if (!s || !sd || !token || (!generated && n_generated > 0)) return fail(FL_ERR_ARG, "null argument");
    if (s->group) return fl_sample(s->ranks[0], sd, generated, n_generated, u, token);
    if (sd->struct_size != (int32_t)sizeof(fl_sampler_desc)) return fail(FL_ERR_ARG, "fl_sampler_desc size mismatch");
    if (!s->built) return fail(FL_ERR_STATE, "tensor-parallel session not connected (fl_session_tp_connect)");
    /* SamplerPipeline's constructor checks (SamplerPipeline.cs:47-48) */
    if (!(sd->temperature >= 0.0f)) return fail(FL_ERR_ARG, "Temperature must be >= 0.");
    if (!(sd->top_p > 0.0f && sd->top_p <= 1.0f)) return fail(FL_ERR_ARG, "topP must be in (0, 1].");
    if (!(sd->repetition_penalty > 0.0f)) return fail(FL_ERR_ARG, "repetition penalty must be > 0");
    if (n_generated < 0) return fail(FL_ERR_ARG, "n_generated must be >= 0");
    const int V = s->m->d.vocab;
    if (cudaSetDevice(s->m->d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    /* (id, occurrences) of the in-range generated ids */
    std::vector<int2> pairs;
    if (sd->repetition_penalty != 1.0f && n_generated > 0) {
        std::vector<int32_t> ids;
        ids.reserve((size_t)n_generated);
        for (int i = 0; i < n_generated; i++)
            if ((uint32_t)generated[i] < (uint32_t)V) ids.push_back(generated[i]);
        std::sort(ids.begin(), ids.end());
        for (size_t i = 0; i < ids.size();) {
            size_t j = i;
            while (j < ids.size() && ids[j] == ids[i]) j++;
            pairs.push_back(make_int2(ids[i], (int)(j - i)));
            i = j;
        }
    }
    if (!s->samp_w) {
        int rc = dalloc(s->allocs, &s->samp_w, (size_t)V * 4 + 256);
        if (rc) return rc;
        s->samp_tok = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(s->samp_w) + (size_t)V * 4);
    }
    if (pairs.size() > s->samp_pairs_cap) {
        const size_t cap = std::max(pairs.size(), std::max<size_t>(256, 2 * s->samp_pairs_cap));
        int rc = dalloc(s->allocs, &s->samp_pairs, cap * sizeof(int2));
        if (rc) return rc;
        s->samp_pairs_cap = cap;
    }
    CK(cudaMemcpyAsync(s->samp_w, s->logits, (size_t)V * 4, cudaMemcpyDeviceToDevice, s->st));
    if (!pairs.empty()) {
        CK(cudaMemcpyAsync(s->samp_pairs, pairs.data(), pairs.size() * sizeof(int2), cudaMemcpyHostToDevice, s->st));
        CK(fl_launch_sample_penalty(s->samp_w, s->samp_pairs, (int)pairs.size(), sd->repetition_penalty, s->st));
    }
    const bool greedy = sd->temperature == 0.0f;
    if (!greedy) {
        if (sd->temperature != 1.0f) CK(fl_launch_sample_scale(s->samp_w, V, 1.0f / sd->temperature, s->st));
        if (sd->top_k > 0 && sd->top_k < V) {
            CK(fl_launch_topk(s->samp_w, V, sd->top_k, s->topk_ids, s->topk_vals, s->topk_scratch,
                              s->topk_scratch_bytes, s->st));
            CK(fl_launch_sample_topk_mask(s->samp_w, V, s->topk_vals, sd->top_k, s->st));
        }
    }
    CK(fl_launch_sample_finish(s->samp_w, V, greedy ? 1 : 0, sd->top_p, u, s->samp_tok, s->st));
    CK(cudaMemcpyAsync(token, s->samp_tok, 4, cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
    return FL_OK;
}

extern "C" int fl_topk_device(const float* logits, int32_t n, int32_t k, int32_t* ids, float* vals, void* stream)
{
    if (!logits || !ids || !vals) return fail(FL_ERR_ARG, "null argument");
    if (n < 1 || n > FL_TOPK_DEVICE_MAX_N)
        return fail(FL_ERR_ARG, "n = %d is outside [1, %d], the size of the static top-k scratch", n,
                    FL_TOPK_DEVICE_MAX_N);
    if (k < 1 || k > n) return fail(FL_ERR_ARG, "k must be in [1, %d]", n);
    CK(fl_launch_topk_static(logits, n, k, ids, vals, static_cast<cudaStream_t>(stream)));
    return FL_OK;
}

/* ── the prompt path ────────────────────────────────────────────────────── */

/* Y[n x N] (fp32, row-major, ld N) = alpha * X[n x K] · W[N x K]^T + beta * Y
 * (fp16, row-major, leading dimensions ldw / ldx, default K) on the tcgen05
 * tensor cores (fl_tc_gemm), `batch` times with the given element strides. */
struct TcOpts {
    int ksplit = 1;
    float* part = nullptr;
    int causal = 0, c_grp = 1, c_start = 0, c_seg = 0, c_seglen = 0;
};

static int tc_gemm(fl_session* s, const __half* W, const __half* X, float* Y, int N, int K, int n, float alpha,
                   int batch = 1, int64_t sW = 0, int64_t sX = 0, int64_t sY = 0, int ldw = 0, int ldx = 0,
                   float beta = 0.0f, const TcOpts& o = TcOpts())
{
    if (!ldw) ldw = K;
    if (!ldx) ldx = K;
    if (batch > 1 && ((sW % ldw) || (sX % ldx))) return fail(FL_ERR_ARG, "GEMM batch strides are not whole rows");
    FlTcGemm p;
    p.M = N;
    p.N = n;
    p.K = K;
    p.batch = batch;
    p.a_batch_rows = batch > 1 ? (int)(sW / ldw) : N;
    p.b_batch_rows = batch > 1 ? (int)(sX / ldx) : n;
    p.Y = Y;
    p.ldy = N;
    p.y_batch = sY;
    p.alpha = alpha;
    p.beta = beta;
    p.err = s->state + ST_ERR;
    p.ksplit = o.ksplit;
    p.part = o.part;
    p.causal = o.causal;
    p.c_grp = o.c_grp;
    p.c_start = o.c_start;
    p.c_seg = o.c_seg;
    p.c_seglen = o.c_seglen;
    CK(fl_tc_gemm(W, ldw, X, ldx, p, s->st));
    return FL_OK;
}

static int pf_gemm(fl_session* s, const __half* W, const __half* X, float* Y, int N, int K0, int n)
{
    return tc_gemm(s, W, X, Y, N, 3 * K0, n, 1.0f / FL_PF_WSCALE);
}

/* split-fp16 weights of a raw matrix into dst (rows x 3*cols) */
static int pf_dequant(fl_session* s, const RawMatrix& r, __half* dst)
{
    CK(fl_launch_dequant_split(r.type, r.d, r.rows, r.cols, dst, s->st, 0, s->state + ST_ERR));
    return FL_OK;
}

/* the same as [lo | hi] rows (rows x 2*cols), the batched steps' layout */
static int bt_dequant(fl_session* s, const RawMatrix& r, __half* dst)
{
    CK(fl_launch_dequant_split(r.type, r.d, r.rows, r.cols, dst, s->st, 1, s->state + ST_ERR));
    return FL_OK;
}

static int pf_alloc(fl_session* s)
{
    fl_model* m = s->m;
    const fl_model_desc& d = m->d;
    const int h = d.hidden, qd = m->qd_l, kvd = m->kvd_l, F = m->ffn_l;
    /* scores and split probabilities take 10 bytes per (query head, key) of
     * a chunk row: the chunk shrinks so they stay within 4 GiB */
    const int nkmax = (s->max_ctx + 63) & ~63;
    const size_t per_tok = (size_t)m->nh_l * nkmax * 10;
    int cap = std::min(s->max_ctx, 2048);
    if ((size_t)cap * per_tok > ((size_t)4 << 30)) cap = std::max(16, (int)((((size_t)4 << 30) / per_tok) & ~(size_t)15));
    if (m->T > 1) cap = std::min(cap, s->pf_tp_rows);
    size_t wmax = std::max({(size_t)(qd + 2 * kvd) * h, (size_t)h * qd, (size_t)2 * F * h, (size_t)h * F});
    if (s->n_slots > 1) wmax = std::max(wmax, (size_t)d.vocab * h); /* the LM head of batched steps */
    const size_t amax = std::max({(size_t)h, (size_t)qd, (size_t)F});
    const size_t ymax = std::max((size_t)h, (size_t)2 * F);
    int rc = FL_OK;
#define AL(p, b) if (!rc) rc = dalloc(s->allocs, &(p), (b))
    AL(s->pf_tokens, (size_t)cap * 4);
    AL(s->pf_x, (size_t)cap * h * 4);
    AL(s->pf_qkv, (size_t)cap * (qd + 2 * kvd) * 4);
    AL(s->pf_q, (size_t)cap * qd * 4);
    AL(s->pf_y, (size_t)cap * ymax * 4);
    AL(s->pf_act, (size_t)cap * amax * 3 * 2);
    AL(s->pf_w, wmax * 3 * 2);
    AL(s->pf_qs, (size_t)cap * qd * 3 * 2);
    AL(s->pf_ks, (size_t)nkmax * kvd * 3 * 2);
    AL(s->pf_vt, (size_t)nkmax * kvd * 3 * 2);
    AL(s->pf_s, (size_t)cap * m->nh_l * nkmax * 4);
    AL(s->pf_p, (size_t)cap * m->nh_l * nkmax * 3 * 2);
    AL(s->pf_o, (size_t)cap * qd * 4);
    s->pf_nkmax = nkmax;
#undef AL
    if (rc) return rc;
    s->pf_cap = cap;
    return FL_OK;
}

/* Where a row-parallel projection writes: pf_y on one GPU; with tensor
 * parallelism this rank's slot of the next exchange (its own memory, which
 * the peers read). */
static float* pf_partial(fl_session* s)
{
    if (s->m->T == 1) return s->pf_y;
    const int parity = (s->pf_epoch + 1) & 1;
    return reinterpret_cast<float*>(s->xchg + s->xchg_pf_off) + (size_t)parity * s->pf_tp_rows * s->m->d.hidden;
}

/* The allreduce of a row-parallel projection's [n x hidden] partial sums
 * (the decode path's TP_REDUCE, for a chunk): raise this rank's flag on every
 * peer with the next epoch, then wait (bounded) for every rank's flag and sum
 * the ranks' slots in rank order into pf_y, identically on every rank. */
static int pf_allreduce(fl_session* s, int n)
{
    fl_model* m = s->m;
    if (m->T == 1) return FL_OK;
    const int epoch = ++s->pf_epoch, parity = epoch & 1;
    const size_t slot_off = s->xchg_pf_off + (size_t)parity * s->pf_tp_rows * m->d.hidden * 4;
    const float* slots[FL_TP_MAX];
    int* flags[FL_TP_MAX];
    for (int q = 0; q < m->T; q++) {
        slots[q] = reinterpret_cast<const float*>(s->tp_peer[q] + slot_off);
        flags[q] = reinterpret_cast<int*>(s->tp_peer[q] + FL_TP_FLAGS_OFF);
    }
    CK(fl_launch_tp_prefill_reduce(slots, flags, m->T, m->rank, epoch, (size_t)n * m->d.hidden, s->pf_y,
                                   s->state + ST_ERR, s->st));
    return FL_OK;
}

/* One chunk of prompt tokens through every layer (the K/V of its positions
 * land in the session's cache). */
static int pf_chunk(fl_session* s, int slot, const int32_t* tokens, int n, int start)
{
    fl_model* m = s->m;
    const fl_model_desc& d = m->d;
    const int h = d.hidden, qd = m->qd_l, kvd = m->kvd_l, F = m->ffn_l, hd = d.head_dim;
    const bool gemma = d.arch == FL_ARCH_GEMMA2;
    const float eps = gemma ? 1e-6f : d.rms_eps;
    int rc = FL_OK;
    CK(cudaMemcpyAsync(s->pf_tokens, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, s->st));
    CK(fl_launch_embed_rows(m->emb_type, m->emb_raw, s->pf_tokens, n, h, d.vocab, s->pf_x, s->state + ST_ERR, s->st));
    for (int l = 0; l < d.n_layers; l++) {
        Layer& L = m->layers[(size_t)l];
        /* residual of the previous FFN (Gemma: its post-norm first), then the attention norm */
        const float* prev = l > 0 ? s->pf_y : nullptr;
        const float* prev_post = l > 0 && gemma ? m->layers[(size_t)l - 1].post_ffn_norm : nullptr;
        CK(fl_launch_rows_norm(s->pf_x, prev, prev_post, L.attn_norm, n, h, eps, gemma, s->pf_act, s->st, 0, nullptr,
                               s->state + ST_ERR));
        /* q, k, v */
        if ((rc = pf_dequant(s, L.rq, s->pf_w))) return rc;
        if ((rc = pf_dequant(s, L.rk, s->pf_w + (size_t)qd * 3 * h))) return rc;
        if ((rc = pf_dequant(s, L.rv, s->pf_w + (size_t)(qd + kvd) * 3 * h))) return rc;
        if ((rc = pf_gemm(s, s->pf_w, s->pf_act, s->pf_qkv, qd + 2 * kvd, h, n))) return rc;
        float* kc = s->kc + (size_t)slot * s->slot_stride + (size_t)l * s->max_ctx * kvd;
        float* vc = s->vc + (size_t)slot * s->slot_stride + (size_t)l * s->max_ctx * kvd;
        CK(fl_launch_rope_kv(s->pf_qkv, L.bq, L.bk, L.bv, m->rope_cs, start, n, qd, kvd, hd, s->pf_q, kc, vc, s->st));
        int window = INT_MAX;
        if (d.arch == FL_ARCH_MISTRAL) window = d.sliding_window;
        if (gemma && (l % 2) == 0) window = d.sliding_window; /* Gemma2ForwardPass.cs:87 */
        if (window <= 0) window = INT_MAX;
        if (l == d.n_layers - 1) break; /* the prompt's last-layer outputs feed nothing: only its K/V are kept */
        {
            /* keys padded to a multiple of 64: the PV product cuts each of its
             * three K segments to the keys a query row may see */
            const int nkv = m->nkv_l, grp = m->nh_l / nkv, nk = start + n, nkp = (nk + 63) & ~63, rows = n * grp;
            TcOpts qk, pv;
            qk.causal = 1;
            qk.c_grp = grp;
            qk.c_start = start;
            pv.causal = 2;
            pv.c_grp = grp;
            pv.c_start = start;
            pv.c_seg = 3;
            pv.c_seglen = nkp;
            CK(fl_launch_attn_q_split(s->pf_q, n, m->nh_l, nkv, hd, s->pf_qs, s->st, s->state + ST_ERR));
            CK(fl_launch_attn_kv_split(kc, vc, nk, nkp, kvd, hd, s->pf_ks, s->pf_vt, s->st, s->state + ST_ERR));
            if ((rc = tc_gemm(s, s->pf_ks, s->pf_qs, s->pf_s, nkp, 3 * hd, rows, 1.0f, nkv, (int64_t)nkp * 3 * hd,
                              (int64_t)rows * 3 * hd, (int64_t)rows * nkp, 0, 0, 0.0f, qk)))
                return rc;
            CK(fl_launch_attn_softmax(s->pf_s, nkv * rows, n, grp, nkp, start, window, d.attn_scale,
                                      gemma ? d.attn_softcap : 0.0f, s->pf_p, s->st));
            if ((rc = tc_gemm(s, s->pf_vt, s->pf_p, s->pf_o, hd, 3 * nkp, rows, 1.0f / 1024.0f, nkv,
                              (int64_t)hd * 3 * nkp, (int64_t)rows * 3 * nkp, (int64_t)rows * hd, 0, 0, 0.0f, pv)))
                return rc;
            CK(fl_launch_attn_out(s->pf_o, n, m->nh_l, nkv, hd, s->pf_act, s->st, s->state + ST_ERR));
        }
        /* output projection, residual (Gemma: post-attention norm), FFN norm */
        if ((rc = pf_dequant(s, L.ro, s->pf_w))) return rc;
        if ((rc = pf_gemm(s, s->pf_w, s->pf_act, pf_partial(s), h, qd, n))) return rc;
        if ((rc = pf_allreduce(s, n))) return rc;
        CK(fl_launch_rows_norm(s->pf_x, s->pf_y, gemma ? L.post_attn_norm : nullptr, L.ffn_norm, n, h, eps, gemma,
                               s->pf_act, s->st, 0, nullptr, s->state + ST_ERR));
        /* gate and up stacked: columns [0, F) gate, [F, 2F) up */
        if ((rc = pf_dequant(s, L.rgate, s->pf_w))) return rc;
        if ((rc = pf_dequant(s, L.rup, s->pf_w + (size_t)F * 3 * h))) return rc;
        if ((rc = pf_gemm(s, s->pf_w, s->pf_act, s->pf_y, 2 * F, h, n))) return rc;
        CK(fl_launch_glu(s->pf_y, n, F, gemma ? 1 : 0, s->pf_act, s->st, 0, nullptr, s->state + ST_ERR));
        if ((rc = pf_dequant(s, L.rdown, s->pf_w))) return rc;
        if ((rc = pf_gemm(s, s->pf_w, s->pf_act, pf_partial(s), h, F, n))) return rc;
        if ((rc = pf_allreduce(s, n))) return rc;
    }
    return FL_OK;
}

/* fl_prefill; with ms != null the chunk loop is bracketed by CUDA events on
 * the session stream and their elapsed time is returned (benchmark hook). */
static int& slot_length(fl_session* s, int slot) { return slot == 0 ? s->cur_len : s->slot_len[(size_t)slot]; }

static int check_prefill(fl_session* s, int slot, const int32_t* tokens, int32_t n, int32_t start_pos)
{
    if (!s->built) return fail(FL_ERR_STATE, "tensor-parallel session not connected (fl_session_tp_connect)");
    const fl_model_desc& d = s->m->d;
    if (slot < 0 || slot >= s->n_slots) return fail(FL_ERR_ARG, "sequence slot %d outside [0, %d)", slot, s->n_slots);
    const int have = slot_length(s, slot);
    if (n < 0 || start_pos < 0 || start_pos > have || start_pos + n > s->max_ctx)
        return fail(FL_ERR_ARG, "prompt positions [%d, %d) do not fit the KV cache (holds %d of %d)", start_pos,
                    start_pos + n, have, s->max_ctx);
    for (int i = 0; i < n; i++)
        if ((uint32_t)tokens[i] >= (uint32_t)d.vocab)
            return fail(FL_ERR_ARG, "Token id %d is outside the valid vocabulary range [0, %d].", tokens[i], d.vocab - 1);
    return FL_OK;
}

static int prefill_impl(fl_session* s, int slot, const int32_t* tokens, int32_t n, int32_t start_pos, float* ms)
{
    if (!s || (!tokens && n)) return fail(FL_ERR_ARG, "null argument");
    if (s->group) {
        if (slot != 0) return fail(FL_ERR_UNSUPPORTED, "batched decode runs on one GPU (tp_size 1)");
        int rc = check_prefill(s->ranks[0], 0, tokens, n, start_pos);
        if (rc || n == 0) return rc;
        /* every rank's prompt buffers first: a rank that failed to allocate
         * while the others ran would leave them waiting for its exchanges */
        rc = run_ranks(s, [&](int r) {
            fl_session* rs = s->ranks[(size_t)r];
            if (rs->pf_cap) return (int)FL_OK;
            if (cudaSetDevice(rs->m->d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
            return pf_alloc(rs);
        });
        if (rc) return rc;
        std::vector<float> t(s->ranks.size(), 0.0f);
        rc = run_ranks(s, [&](int r) {
            return prefill_impl(s->ranks[(size_t)r], 0, tokens, n, start_pos, ms ? &t[(size_t)r] : nullptr);
        });
        if (!rc && ms) *ms = *std::max_element(t.begin(), t.end());
        return rc;
    }
    int rc = check_prefill(s, slot, tokens, n, start_pos);
    if (rc || n == 0) return rc;
    fl_model* m = s->m;
    const fl_model_desc& d = m->d;
    if (cudaSetDevice(d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    if (!s->pf_cap && (rc = pf_alloc(s))) return rc;
    if (m->T > 1) CK(cudaMemcpy(&s->pf_epoch, s->tp_epoch, 4, cudaMemcpyDeviceToHost)); /* continues the token loop's */
    cudaEvent_t ev[2] = {nullptr, nullptr};
    if (ms) {
        CK(cudaEventCreate(&ev[0]));
        CK(cudaEventCreate(&ev[1]));
        CK(cudaEventRecord(ev[0], s->st));
    }
    for (int c = 0; c < n && !rc; c += s->pf_cap) {
        const int len = std::min(s->pf_cap, n - c);
        rc = pf_chunk(s, slot, tokens + c, len, start_pos + c);
    }
    if (m->T > 1 && !rc && cudaMemcpyAsync(s->tp_epoch, &s->pf_epoch, 4, cudaMemcpyHostToDevice, s->st) != cudaSuccess)
        rc = fail(FL_ERR_CUDA, "epoch update failed");
    if (ms && !rc && cudaEventRecord(ev[1], s->st) != cudaSuccess) rc = fail(FL_ERR_CUDA, "cudaEventRecord failed");
    if (!rc && cudaStreamSynchronize(s->st) != cudaSuccess) rc = fail(FL_ERR_CUDA, "prefill: stream failed");
    if (!rc) rc = check_device_err(s);
    if (ms && !rc && cudaEventElapsedTime(ms, ev[0], ev[1]) != cudaSuccess) rc = fail(FL_ERR_CUDA, "cudaEventElapsedTime failed");
    for (cudaEvent_t e : ev)
        if (e) cudaEventDestroy(e);
    if (rc) {
        /* positions from start_pos on may hold a partial prompt: the cache keeps those before it */
        slot_length(s, slot) = std::min(slot_length(s, slot), (int)start_pos);
        return rc;
    }
    slot_length(s, slot) = start_pos + n;
    return FL_OK;
}

extern "C" int fl_prefill(fl_session* s, const int32_t* tokens, int32_t n, int32_t start_pos)
{
    return prefill_impl(s, 0, tokens, n, start_pos, nullptr);
}

extern "C" int fl_prefill_seq(fl_session* s, int32_t seq_slot, const int32_t* tokens, int32_t n, int32_t start_pos)
{
    return prefill_impl(s, seq_slot, tokens, n, start_pos, nullptr);
}

extern "C" int fl_time_prefill(fl_session* s, const int32_t* tokens, int32_t n, int32_t start_pos, float* ms)
{
    if (!ms) return fail(FL_ERR_ARG, "null argument");
    return prefill_impl(s, 0, tokens, n, start_pos, ms);
}

/* ── batched decode ─────────────────────────────────────────────────────── */

/* The split-fp16 weights of every projection and of the LM head, kept for
 * the session's batched steps as [lo | hi] rows: 4 bytes per weight (8B:
 * ~30 GB), tried once; without them each step dequantizes into the prompt
 * path's buffer. */
static void bt_cache_weights(fl_session* s)
{
    s->bt_cache_tried = true;
    fl_model* m = s->m;
    const fl_model_desc& d = m->d;
    const int h = d.hidden, qd = m->qd_l, kvd = m->kvd_l, F = m->ffn_l;
    std::vector<size_t> sizes;
    for (int l = 0; l < d.n_layers; l++) {
        sizes.push_back((size_t)(qd + 2 * kvd) * h);
        sizes.push_back((size_t)h * qd);
        sizes.push_back((size_t)2 * F * h);
        sizes.push_back((size_t)h * F);
    }
    sizes.push_back((size_t)d.vocab * h);
    size_t total = 0;
    for (size_t e : sizes) total += (e * 2 * 2 + 255) & ~(size_t)255;
    size_t free_b = 0, tot_b = 0;
    if (cudaMemGetInfo(&free_b, &tot_b) != cudaSuccess || total + ((size_t)4 << 30) > free_b) return;
    uint8_t* base = nullptr;
    if (cudaMalloc(&base, total) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    s->allocs.push_back(base);
    size_t off = 0;
    for (size_t e : sizes) {
        s->bt_w.push_back(reinterpret_cast<__half*>(base + off));
        off += (e * 2 * 2 + 255) & ~(size_t)255;
    }
    for (int l = 0; l < d.n_layers; l++) {
        const Layer& L = m->layers[(size_t)l];
        __half** w = &s->bt_w[(size_t)l * 4];
        if (bt_dequant(s, L.rq, w[0]) || bt_dequant(s, L.rk, w[0] + (size_t)qd * 2 * h) ||
            bt_dequant(s, L.rv, w[0] + (size_t)(qd + kvd) * 2 * h) || bt_dequant(s, L.ro, w[1]) ||
            bt_dequant(s, L.rgate, w[2]) || bt_dequant(s, L.rup, w[2] + (size_t)F * 2 * h) ||
            bt_dequant(s, L.rdown, w[3])) {
            s->bt_w.clear();
            return;
        }
    }
    if (bt_dequant(s, m->rout, s->bt_w.back())) s->bt_w.clear();
}

/* K splits of a batched projection with mt weight-row tiles and nkb 64-wide
 * k-blocks: enough work items for two per SM, at least 8 k-blocks each. */
static int bt_ksplit(int mt, int nkb)
{
    int ks = (2 * 148 + mt - 1) / mt;
    ks = std::min(ks, std::max(1, nkb / 8));
    return std::max(1, std::min(ks, 16));
}

/* Y[B x N] = X · W^T for the batched steps, one GEMM over K' = 2K: W as
 * [lo | hi] rows (scaled by FL_PF_WSCALE), X as 2B rows, [hi | hi] for
 * sequence b and [0 | lo] for row B + b.  Rows b get lo*hi + hi*hi (the small
 * term accumulated first), rows B + b get hi*lo; the consumers add the two
 * halves as they read.  Every weight byte is read once, the K range split
 * across CTAs when the weight rows alone make too few work items. */
static int bt_gemm(fl_session* s, const __half* W, const __half* X, float* Y, int N, int K, int B)
{
    TcOpts o;
    o.ksplit = bt_ksplit((N + 127) / 128, (2 * K + 63) / 64);
    o.part = s->bt_part;
    int rc = tc_gemm(s, W, X, s->bt_y2, N, 2 * K, 2 * B, 1.0f / FL_PF_WSCALE, 1, 0, 0, 0, 2 * K, 2 * K, 0.0f, o);
    if (rc) return rc;
    if (Y) CK(fl_launch_add_halves(s->bt_y2, B, N, Y, s->st));
    return FL_OK;
}

extern "C" int fl_forward_batch(fl_session* s, int32_t B, const int32_t* tokens, const int32_t* positions,
                                const int32_t* slots, float* logits, int32_t* argmax)
{
    if (!s || !tokens || !positions || !slots) return fail(FL_ERR_ARG, "null argument");
    if (s->group) return fail(FL_ERR_UNSUPPORTED, "batched decode runs on one GPU (tp_size 1)");
    if (!s->built) return fail(FL_ERR_STATE, "tensor-parallel session not connected (fl_session_tp_connect)");
    fl_model* m = s->m;
    const fl_model_desc& d = m->d;
    if (m->T > 1) return fail(FL_ERR_UNSUPPORTED, "batched decode runs on one GPU (tp_size 1)");
    if (B < 1 || B > s->n_slots) return fail(FL_ERR_ARG, "batch %d outside [1, %d] (the session's sequence slots)", B,
                                             s->n_slots);
    std::vector<char> seen((size_t)s->n_slots, 0);
    for (int b = 0; b < B; b++) {
        if (slots[b] < 0 || slots[b] >= s->n_slots)
            return fail(FL_ERR_ARG, "sequence slot %d outside [0, %d)", slots[b], s->n_slots);
        if (seen[(size_t)slots[b]]++) return fail(FL_ERR_ARG, "sequence slot %d appears twice in one batch", slots[b]);
        if ((uint32_t)tokens[b] >= (uint32_t)d.vocab)
            return fail(FL_ERR_ARG, "Token id %d is outside the valid vocabulary range [0, %d].", tokens[b], d.vocab - 1);
        if (positions[b] < 0 || positions[b] >= s->max_ctx || positions[b] > slot_length(s, slots[b]))
            return fail(FL_ERR_ARG, "position %d of slot %d skips cached positions or exceeds the context", positions[b],
                        slots[b]);
    }
    if (cudaSetDevice(d.device) != cudaSuccess) return fail(FL_ERR_CUDA, "cudaSetDevice failed");
    int rc = FL_OK;
    if (!s->pf_cap && (rc = pf_alloc(s))) return rc;
    if (4 * B > 3 * s->pf_cap) /* 2B stacked rows of 2K halves in the prompt path's buffer of cap rows of 3K */
        return fail(FL_ERR_UNSUPPORTED, "batch %d above %d rows (3/4 of the prompt path's)", B, 3 * s->pf_cap / 4);
    const int h = d.hidden, qd = m->qd_l, kvd = m->kvd_l, F = m->ffn_l, hd = d.head_dim;
    if (!s->bt_pos) {
        const int S = s->n_slots;
        const size_t widest = std::max({(size_t)(qd + 2 * kvd), (size_t)h, (size_t)2 * F, (size_t)d.vocab});
        if ((rc = dalloc(s->allocs, &s->bt_pos, (size_t)S * 4)) || (rc = dalloc(s->allocs, &s->bt_slot, (size_t)S * 4)) ||
            (rc = dalloc(s->allocs, &s->bt_argmax, (size_t)S * 4)) ||
            (rc = dalloc(s->allocs, &s->bt_logits, (size_t)S * d.vocab * 4)) ||
            (rc = dalloc(s->allocs, &s->bt_y2, (size_t)2 * S * widest * 4)))
            return rc;
        /* the largest K-split partial buffer of any projection */
        size_t part = 0;
        const int shapes[5][2] = {{qd + 2 * kvd, h}, {h, qd}, {2 * F, h}, {h, F}, {d.vocab, h}};
        for (auto& sh : shapes)
            part = std::max(part, (size_t)bt_ksplit((sh[0] + 127) / 128, (2 * sh[1] + 63) / 64) * 2 * S * sh[0]);
        if ((rc = dalloc(s->allocs, &s->bt_part, part * 4))) return rc;
    }
    if (!s->bt_cache_tried) bt_cache_weights(s);
    const bool cached = !s->bt_w.empty();
    const bool gemma = d.arch == FL_ARCH_GEMMA2;
    const float eps = gemma ? 1e-6f : d.rms_eps;
    /* activations are stacked for bt_gemm: B [hi | hi] rows, then B [0 | lo] rows */
    const int stk = B;
    CK(cudaMemcpyAsync(s->pf_tokens, tokens, (size_t)B * 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaMemcpyAsync(s->bt_pos, positions, (size_t)B * 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaMemcpyAsync(s->bt_slot, slots, (size_t)B * 4, cudaMemcpyHostToDevice, s->st));
    CK(fl_launch_embed_rows(m->emb_type, m->emb_raw, s->pf_tokens, B, h, d.vocab, s->pf_x, s->state + ST_ERR, s->st));
    for (int l = 0; l < d.n_layers; l++) {
        Layer& L = m->layers[(size_t)l];
        __half* const* cw = cached ? &s->bt_w[(size_t)l * 4] : nullptr;
        /* a projection's output stays as the two halves in bt_y2 ([B][N], then
         * [B][N]); the next kernel adds them as it reads */
        const float* prev = l > 0 ? s->bt_y2 : nullptr;
        const float* prev_lo = l > 0 ? s->bt_y2 + (size_t)B * h : nullptr;
        const float* prev_post = l > 0 && gemma ? m->layers[(size_t)l - 1].post_ffn_norm : nullptr;
        CK(fl_launch_rows_norm(s->pf_x, prev, prev_post, L.attn_norm, B, h, eps, gemma, s->pf_act, s->st, stk, prev_lo,
                               s->state + ST_ERR));
        const __half* w = cached ? cw[0] : s->pf_w;
        if (!cached && ((rc = bt_dequant(s, L.rq, s->pf_w)) || (rc = bt_dequant(s, L.rk, s->pf_w + (size_t)qd * 2 * h)) ||
                        (rc = bt_dequant(s, L.rv, s->pf_w + (size_t)(qd + kvd) * 2 * h))))
            return rc;
        if ((rc = bt_gemm(s, w, s->pf_act, nullptr, qd + 2 * kvd, h, B))) return rc;
        float* kc = s->kc + (size_t)l * s->max_ctx * kvd;
        float* vc = s->vc + (size_t)l * s->max_ctx * kvd;
        CK(fl_launch_rope_kv_rows(s->bt_y2, L.bq, L.bk, L.bv, m->rope_cs, s->bt_pos, s->bt_slot, s->slot_stride, B, qd,
                                  kvd, hd, s->pf_q, kc, vc, s->st, s->bt_y2 + (size_t)B * (qd + 2 * kvd)));
        int window = INT_MAX;
        if (d.arch == FL_ARCH_MISTRAL) window = d.sliding_window;
        if (gemma && (l % 2) == 0) window = d.sliding_window; /* Gemma2ForwardPass.cs:87 */
        if (window <= 0) window = INT_MAX;
        CK(fl_launch_batch_attn(s->pf_q, kc, vc, s->bt_pos, s->bt_slot, s->slot_stride, B, m->nh_l, m->nkv_l, hd, window,
                                d.attn_scale, gemma ? d.attn_softcap : 0.0f, s->pf_act, s->st, stk, s->state + ST_ERR));
        w = cached ? cw[1] : s->pf_w;
        if (!cached && (rc = bt_dequant(s, L.ro, s->pf_w))) return rc;
        if ((rc = bt_gemm(s, w, s->pf_act, nullptr, h, qd, B))) return rc;
        CK(fl_launch_rows_norm(s->pf_x, s->bt_y2, gemma ? L.post_attn_norm : nullptr, L.ffn_norm, B, h, eps, gemma,
                               s->pf_act, s->st, stk, s->bt_y2 + (size_t)B * h, s->state + ST_ERR));
        w = cached ? cw[2] : s->pf_w;
        if (!cached && ((rc = bt_dequant(s, L.rgate, s->pf_w)) || (rc = bt_dequant(s, L.rup, s->pf_w + (size_t)F * 2 * h))))
            return rc;
        if ((rc = bt_gemm(s, w, s->pf_act, nullptr, 2 * F, h, B))) return rc;
        CK(fl_launch_glu(s->bt_y2, B, F, gemma ? 1 : 0, s->pf_act, s->st, stk, s->bt_y2 + (size_t)B * 2 * F,
                         s->state + ST_ERR));
        w = cached ? cw[3] : s->pf_w;
        if (!cached && (rc = bt_dequant(s, L.rdown, s->pf_w))) return rc;
        if ((rc = bt_gemm(s, w, s->pf_act, nullptr, h, F, B))) return rc;
    }
    /* final norm (after the last residual) and the LM head */
    CK(fl_launch_rows_norm(s->pf_x, s->bt_y2, gemma ? m->layers.back().post_ffn_norm : nullptr, m->out_norm, B, h, eps,
                           gemma, s->pf_act, s->st, stk, s->bt_y2 + (size_t)B * h, s->state + ST_ERR));
    const __half* wh = cached ? s->bt_w.back() : s->pf_w;
    if (!cached && (rc = bt_dequant(s, m->rout, s->pf_w))) return rc;
    if ((rc = bt_gemm(s, wh, s->pf_act, s->bt_logits, d.vocab, h, B))) return rc;
    if (gemma && d.final_softcap > 0.0f) CK(fl_launch_softcap_rows(s->bt_logits, (size_t)B * d.vocab, d.final_softcap, s->st));
    CK(fl_launch_argmax_rows(s->bt_logits, B, d.vocab, s->bt_argmax, s->st));
    if (argmax) CK(cudaMemcpyAsync(argmax, s->bt_argmax, (size_t)B * 4, cudaMemcpyDeviceToHost, s->st));
    if (logits) CK(cudaMemcpyAsync(logits, s->bt_logits, (size_t)B * d.vocab * 4, cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
    if ((rc = check_device_err(s))) return rc;
    for (int b = 0; b < B; b++) slot_length(s, slots[b]) = positions[b] + 1;
    return FL_OK;
}

/* ── stateless helpers ──────────────────────────────────────────────────── */
extern "C" int fl_dequant(int32_t type, const void* src, uint64_t nbytes, float* dst, uint64_t dst_len)
{
    /* Dequantizer.Dequantize (Dequantizer.cs:488-504) validation order */
    int be = block_elems(type), bb = block_bytes(type);
    if (!be) return fail(FL_ERR_UNSUPPORTED, "Tensor type %d is not supported for dequantization.", type);
    if (nbytes % (uint64_t)bb) return fail(FL_ERR_ARG, "Source length must be a multiple of %d.", bb);
    uint64_t n = nbytes / bb * be;
    if (dst_len < n) return fail(FL_ERR_ARG, "Destination must hold at least %llu floats.", (unsigned long long)n);
    if (n == 0) return FL_OK;
    if (!src || !dst) return fail(FL_ERR_ARG, "null argument");
    uint8_t* dsrc = nullptr;
    float* ddst = nullptr;
    CK(cudaMalloc(&dsrc, nbytes));
    cudaError_t e = cudaMalloc(&ddst, n * 4);
    if (e != cudaSuccess) {
        cudaFree(dsrc);
        return fail(FL_ERR_OOM, "cudaMalloc: %s", cudaGetErrorString(e));
    }
    e = cudaMemcpy(dsrc, src, nbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = fl_launch_dequant(type, dsrc, (int64_t)n, ddst, 0);
    if (e == cudaSuccess) e = cudaMemcpy(dst, ddst, n * 4, cudaMemcpyDeviceToHost);
    cudaFree(dsrc);
    cudaFree(ddst);
    if (e != cudaSuccess) return fail(FL_ERR_CUDA, "fl_dequant: %s", cudaGetErrorString(e));
    return FL_OK;
}

/* Test hook (internal): the prefill's split-fp16 weight layout of a raw
 * matrix, rows x 3*cols halves ([hi | lo | hi] of value * FL_PF_WSCALE; values
 * past the fp16 range are written as they fall, without the range flag). */
extern "C" int fl_dequant_split_test(int32_t type, const void* src, uint64_t nbytes, int32_t rows, int32_t cols,
                                     uint16_t* dst)
{
    if (!src || !dst || rows <= 0 || cols <= 0) return fail(FL_ERR_ARG, "bad argument");
    const int be = block_elems(type), bb = block_bytes(type);
    if (!be || cols % be) return fail(FL_ERR_ARG, "cols must be whole blocks");
    if ((uint64_t)rows * cols / be * bb != nbytes) return fail(FL_ERR_ARG, "byte size mismatch");
    uint8_t* d_src = nullptr;
    __half* d_dst = nullptr;
    const size_t out_bytes = (size_t)rows * cols * 3 * 2;
    CK(cudaMalloc(&d_src, nbytes));
    cudaError_t e = cudaMalloc(&d_dst, out_bytes);
    if (e == cudaSuccess) e = cudaMemcpy(d_src, src, nbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = fl_launch_dequant_split(type, d_src, rows, cols, d_dst, 0);
    if (e == cudaSuccess) e = cudaMemcpy(dst, d_dst, out_bytes, cudaMemcpyDeviceToHost);
    cudaFree(d_src);
    if (d_dst) cudaFree(d_dst);
    if (e != cudaSuccess) return fail(FL_ERR_CUDA, "fl_dequant_split_test: %s", cudaGetErrorString(e));
    return FL_OK;
}

extern "C" int fl_gemm_f16(const void* a, int64_t lda, const void* b, int64_t ldb, int32_t M, int32_t N, int32_t K,
                           int32_t batch, int32_t a_batch_rows, int32_t b_batch_rows, float alpha, float beta,
                           int32_t ksplit, int32_t causal, int32_t c_grp, int32_t c_start, int32_t c_seg, float* y)
{
    if (!a || !b || !y) return fail(FL_ERR_ARG, "null argument");
    if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || lda < K || ldb < K || (lda % 8) || (ldb % 8))
        return fail(FL_ERR_ARG, "bad GEMM shape (M %d, N %d, K %d, lda %lld, ldb %lld: strides multiples of 8)", M, N,
                    K, (long long)lda, (long long)ldb);
    if (batch > 1 && (a_batch_rows < M || b_batch_rows < N)) return fail(FL_ERR_ARG, "batch rows below M / N");
    if (ksplit < 1 || ksplit > 64 || causal < 0 || causal > 2 || (ksplit > 1 && causal) || (causal && c_grp < 1) ||
        (causal == 2 && (c_seg < 1 || K % c_seg || (K / c_seg) % 64)))
        return fail(FL_ERR_ARG, "bad split / causal arguments");
    const long long arows = batch > 1 ? (long long)batch * a_batch_rows : M;
    const long long brows = batch > 1 ? (long long)batch * b_batch_rows : N;
    const size_t ab = (size_t)arows * lda * 2, bb = (size_t)brows * ldb * 2, yb = (size_t)batch * N * M * 4;
    std::vector<void*> al;
    __half *da = nullptr, *db = nullptr;
    float* dy = nullptr;
    int* derr = nullptr;
    float* dpart = nullptr;
    int rc = dalloc(al, &da, ab);
    if (!rc) rc = dalloc(al, &db, bb);
    if (!rc) rc = dalloc(al, &dy, yb);
    if (!rc) rc = dalloc(al, &derr, 16);
    if (!rc && ksplit > 1) rc = dalloc(al, &dpart, yb * (size_t)ksplit);
    cudaError_t e = cudaSuccess;
    if (!rc) {
        e = cudaMemcpy(da, a, ab, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(db, b, bb, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(dy, y, yb, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemset(derr, 0, 16);
        if (e == cudaSuccess) {
            FlTcGemm p;
            p.M = M;
            p.N = N;
            p.K = K;
            p.batch = batch;
            p.a_batch_rows = batch > 1 ? a_batch_rows : M;
            p.b_batch_rows = batch > 1 ? b_batch_rows : N;
            p.Y = dy;
            p.ldy = M;
            p.y_batch = (long long)N * M;
            p.alpha = alpha;
            p.beta = beta;
            p.err = derr;
            p.ksplit = ksplit;
            p.part = dpart;
            p.causal = causal;
            p.c_grp = c_grp;
            p.c_start = c_start;
            p.c_seg = c_seg;
            p.c_seglen = causal == 2 ? K / c_seg : 0;
            e = fl_tc_gemm(da, lda, db, ldb, p, 0);
        }
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        int herr = 0;
        if (e == cudaSuccess) e = cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(y, dy, yb, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && herr) rc = fail(FL_ERR_TIMEOUT, "a bounded wait of the GEMM expired");
        if (e != cudaSuccess) rc = fail(FL_ERR_CUDA, "fl_gemm_f16: %s", cudaGetErrorString(e));
    }
    for (void* p : al) cudaFree(p);
    return rc;
}

extern "C" int fl_matvec(int32_t type, const void* w, uint64_t nbytes, int32_t rows, int32_t cols, const float* x,
                         float* y)
{
    if (!w || !x || !y) return fail(FL_ERR_ARG, "null argument");
    fl_matrix_layout L;
    int r = fl_layout_for(type, rows, cols, &L);
    if (r == -1) return fail(FL_ERR_UNSUPPORTED, "type %d has no quantized matvec path", type);
    if (r == -2) return fail(FL_ERR_UNSUPPORTED, "row length %d is not a multiple of 32", cols);
    if ((int64_t)nbytes != L.gguf_bytes) return fail(FL_ERR_ARG, "byte length does not match rows x cols");
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    std::vector<uint8_t> host((size_t)L.total_bytes);
    fl_repack(&L, static_cast<const uint8_t*>(w), nullptr, nullptr, host.data(), 0);
    float amax = 0.0f;
    for (int i = 0; i < cols; i++) amax = fmaxf(amax, fabsf(x[i]));
    std::vector<void*> al;
    DevMatrix dm;
    dm.L = L;
    float *dx = nullptr, *dy = nullptr, *dam = nullptr;
    int* derr = nullptr;
    int rc = dalloc(al, &dm.d, (size_t)L.total_bytes);
    if (!rc) rc = dalloc(al, &dx, (size_t)L.n_kb * 256 * 4);
    if (!rc) rc = dalloc(al, &dy, (size_t)rows * 4);
    if (!rc) rc = dalloc(al, &dam, 16);
    if (!rc) rc = dalloc(al, &derr, 16);
    cudaError_t e = cudaSuccess;
    if (!rc) {
        e = cudaMemcpy(dm.d, host.data(), (size_t)L.total_bytes, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(dx, x, (size_t)cols * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(dam, &amax, 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemset(derr, 0, 16);
        if (e == cudaSuccess) {
            FlMvArgs a = base_args(nullptr, dm, cols);
            fl_mv_ring_config(a);
            a.err = derr;
            a.in_mode = FL_IN_PLAIN;
            a.x = dx;
            a.absmax = dam;
            a.epi = FL_EPI_STORE;
            a.y = dy;
            int grid = a.n_tiles < sms ? a.n_tiles : sms;
            e = fl_launch_matvec(a, grid, 0, false);
        }
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemcpy(y, dy, (size_t)rows * 4, cudaMemcpyDeviceToHost);
        int err = 0;
        if (e == cudaSuccess) e = cudaMemcpy(&err, derr, 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && err) rc = fail(FL_ERR_TIMEOUT, "bounded device wait expired");
    }
    for (void* p : al) cudaFree(p);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(FL_ERR_CUDA, "fl_matvec: %s", cudaGetErrorString(e));
    return FL_OK;
}

/* Per-phase device milliseconds of the most recent step (diagnostics; phase
 * order: embed, then per layer qkv, attention, wo, gate/up, down, then head). */
/* Per phase p < n_phases - 1 and CTA b: ms from the phase's start (CTA 0) to
 * the moment CTA b finished its share of it, out[p * grid + b]. */
extern "C" int fl_session_cta_done_ms(fl_session* s, double* out, int64_t cap, int32_t* grid)
{
    if (!s || !out || !grid) return fail(FL_ERR_ARG, "null argument");
    if (s->group) return fail(FL_ERR_UNSUPPORTED, "measurement hook of one rank: not available on a group session");
    const int G = s->tk_grid;
    std::vector<uint64_t> ts((size_t)s->n_phases + 1), done((size_t)s->n_phases * G);
    CK(cudaMemcpy(ts.data(), s->timestamps, ts.size() * 8, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(done.data(), s->cta_done, done.size() * 8, cudaMemcpyDeviceToHost));
    *grid = G;
    for (int p = 0; p + 1 < s->n_phases; p++)
        for (int b = 0; b < G; b++)
            if ((int64_t)p * G + b < cap) out[(size_t)p * G + b] = ((double)done[(size_t)p * G + b] - (double)ts[p]) * 1e-6;
    return FL_OK;
}

/* The raw per-warp matvec counters of CTA 0 (FlTokenArgs.detail) and the
 * phase start stamps: out = [n_phases + 1] starts, then the detail array. */
extern "C" int fl_session_detail(fl_session* s, uint64_t* out, int64_t cap, int32_t* n_phases, int32_t* n_warps)
{
    if (!s || !out || !n_phases || !n_warps) return fail(FL_ERR_ARG, "null argument");
    if (s->group) return fail(FL_ERR_UNSUPPORTED, "measurement hook of one rank: not available on a group session");
    const size_t nd = (size_t)s->n_phases * (FL_TK_WARPS * 4 + 1), nt = (size_t)s->n_phases + 1;
    if ((int64_t)(nd + nt) > cap) return fail(FL_ERR_ARG, "need %zu entries", nd + nt);
    CK(cudaMemcpy(out, s->timestamps, nt * 8, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(out + nt, s->detail, nd * 8, cudaMemcpyDeviceToHost));
    *n_phases = s->n_phases;
    *n_warps = FL_TK_WARPS;
    return FL_OK;
}

extern "C" int fl_session_phase_ms(fl_session* s, double* out, int32_t cap, int32_t* n)
{
    if (!s || !out || !n) return fail(FL_ERR_ARG, "null argument");
    if (s->group) return fail(FL_ERR_UNSUPPORTED, "measurement hook of one rank: not available on a group session");
    std::vector<uint64_t> ts((size_t)s->n_phases + 1);
    CK(cudaMemcpy(ts.data(), s->timestamps, ts.size() * 8, cudaMemcpyDeviceToHost));
    *n = s->n_phases;
    for (int p = 0; p < s->n_phases && p < cap; p++) out[p] = (double)(ts[(size_t)p + 1] - ts[(size_t)p]) * 1e-6;
    return FL_OK;
}

/* ── tensor parallelism driven from one host thread ─────────────────────── */

/* The reference calls Forward from one thread per request
 * (LlamaForwardPass.cs:29).  A group model (tp_rank FL_TP_ALL) keeps one rank
 * model per device, and its sessions run every call on all ranks at once:
 * rank 0 on the calling thread, the others on the session's worker threads.
 * The ranks' kernels wait on one another inside each step, so every rank's
 * launches are issued and waited for concurrently. */

static std::mutex g_layout_mu;
static int g_layout_tp = 0;
static int g_layout_dev[FL_TP_MAX];

extern "C" int fl_init(int32_t tp, const int32_t* devices)
{
    if (tp < 1 || tp > FL_TP_MAX || (tp & (tp - 1))) return fail(FL_ERR_UNSUPPORTED, "tp %d (1, 2, 4 or 8)", tp);
    int dev[FL_TP_MAX];
    for (int r = 0; r < tp; r++) {
        dev[r] = devices ? devices[r] : r;
        if (dev[r] < 0) return fail(FL_ERR_ARG, "device %d", dev[r]);
        for (int q = 0; q < r; q++)
            if (dev[q] == dev[r]) return fail(FL_ERR_ARG, "ranks %d and %d share device %d", q, r, dev[r]);
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return fail(FL_ERR_CUDA, "no CUDA device");
    }
    for (int r = 0; r < tp; r++)
        if (dev[r] >= n) return fail(FL_ERR_ARG, "device %d outside [0, %d)", dev[r], n);
    for (int r = 0; r < tp; r++)
        for (int q = 0; q < tp; q++) {
            int can = 0;
            if (q != r && (cudaDeviceCanAccessPeer(&can, dev[r], dev[q]) != cudaSuccess || !can))
                return fail(FL_ERR_UNSUPPORTED, "device %d cannot access device %d's memory", dev[r], dev[q]);
        }
    std::lock_guard<std::mutex> lk(g_layout_mu);
    g_layout_tp = tp;
    for (int r = 0; r < tp; r++) g_layout_dev[r] = dev[r];
    return FL_OK;
}

static int group_model_create(const fl_model_desc& d, fl_model** out)
{
    const int T = d.tp_size;
    if (T < 2 || T > FL_TP_MAX || (T & (T - 1))) return fail(FL_ERR_UNSUPPORTED, "tp_size %d for a group (2, 4 or 8)", T);
    int dev[FL_TP_MAX];
    {
        std::lock_guard<std::mutex> lk(g_layout_mu);
        if (g_layout_tp && g_layout_tp != T)
            return fail(FL_ERR_STATE, "fl_init set %d ranks, the model asks for %d", g_layout_tp, T);
        for (int r = 0; r < T; r++) dev[r] = g_layout_tp ? g_layout_dev[r] : r;
    }
    fl_model* g = new fl_model();
    g->d = d;
    g->T = T;
    g->group = true;
    for (int r = 0; r < T; r++) {
        fl_model_desc dr = d;
        dr.device = dev[r];
        dr.tp_rank = r;
        fl_model* m = nullptr;
        int rc = fl_model_create(&dr, &m);
        if (rc) {
            std::string msg = g_err;
            fl_model_destroy(g);
            return fail(rc, "rank %d: %s", r, msg.c_str());
        }
        g->ranks.push_back(m);
    }
    *out = g;
    return FL_OK;
}

struct RankPool {
    std::vector<std::thread> th;
    std::mutex mu;
    std::condition_variable go, done;
    const std::function<int(int)>* job = nullptr;
    uint64_t gen = 0;
    int pending = 0;
    bool stop = false;
    std::vector<int> rc;
    std::vector<std::string> msg;
};

static void pool_worker(RankPool* p, int r)
{
    uint64_t seen = 0;
    for (;;) {
        const std::function<int(int)>* job = nullptr;
        {
            std::unique_lock<std::mutex> lk(p->mu);
            p->go.wait(lk, [&] { return p->stop || p->gen != seen; });
            if (p->stop) return;
            seen = p->gen;
            job = p->job;
        }
        const int rc = (*job)(r);
        std::lock_guard<std::mutex> lk(p->mu);
        p->rc[(size_t)r] = rc;
        if (rc) p->msg[(size_t)r] = g_err;
        if (--p->pending == 0) p->done.notify_one();
    }
}

static void pool_stop(RankPool* p)
{
    {
        std::lock_guard<std::mutex> lk(p->mu);
        p->stop = true;
    }
    p->go.notify_all();
    for (std::thread& t : p->th) t.join();
    delete p;
}

/* f(r) on every rank at once; the first failing rank's status and message. */
static int run_ranks(fl_session* s, const std::function<int(int)>& f)
{
    RankPool* p = s->pool;
    const int T = (int)s->ranks.size();
    {
        std::lock_guard<std::mutex> lk(p->mu);
        p->job = &f;
        p->pending = T - 1;
        for (int r = 0; r < T; r++) {
            p->rc[(size_t)r] = 0;
            p->msg[(size_t)r].clear();
        }
        p->gen++;
    }
    p->go.notify_all();
    const int rc0 = f(0);
    const std::string msg0 = rc0 ? g_err : std::string();
    {
        std::unique_lock<std::mutex> lk(p->mu);
        p->done.wait(lk, [&] { return p->pending == 0; });
    }
    if (rc0) return fail(rc0, "rank 0: %s", msg0.c_str());
    for (int r = 1; r < T; r++)
        if (p->rc[(size_t)r]) return fail(p->rc[(size_t)r], "rank %d: %s", r, p->msg[(size_t)r].c_str());
    return FL_OK;
}

static int group_session_create(fl_model* g, int32_t max_ctx, int32_t max_batch, int32_t kv_dtype, fl_session** out)
{
    if (max_batch > 1) return fail(FL_ERR_UNSUPPORTED, "batched sessions run on one GPU (tp_size 1)");
    const int T = g->T;
    fl_session* s = new fl_session();
    s->m = g;
    s->group = true;
    std::vector<uint8_t> handles((size_t)T * FL_TP_HANDLE_BYTES);
    int rc = FL_OK;
    for (int r = 0; r < T && !rc; r++) {
        fl_session* rs = nullptr;
        rc = fl_session_create(g->ranks[(size_t)r], max_ctx, 1, kv_dtype, &rs);
        if (!rc) {
            s->ranks.push_back(rs);
            rc = fl_session_tp_handle(rs, handles.data() + (size_t)r * FL_TP_HANDLE_BYTES);
        }
    }
    for (int r = 0; r < T && !rc; r++) rc = fl_session_tp_connect(s->ranks[(size_t)r], handles.data());
    if (!rc) {
        RankPool* p = new RankPool();
        p->rc.assign((size_t)T, 0);
        p->msg.assign((size_t)T, std::string());
        s->pool = p;
        try {
            for (int r = 1; r < T; r++) p->th.emplace_back(pool_worker, p, r);
        } catch (...) {
            rc = fail(FL_ERR_STATE, "could not start the rank threads");
        }
    }
    if (rc) {
        std::string msg = g_err;
        fl_session_destroy(s);
        return fail(rc, "%s", msg.c_str());
    }
    s->max_ctx = s->ranks[0]->max_ctx;
    *out = s;
    return FL_OK;
}

static void group_session_destroy(fl_session* s)
{
    if (s->pool) pool_stop(s->pool);
    for (fl_session* r : s->ranks) fl_session_destroy(r);
    delete s;
}
