/*
 * fl_misc.cu — the decode-step kernels around the matvecs: bit-exact
 * dequantization (Dequantizer.cs), the embedding row, split-K GQA attention over
 * the HBM KV cache, the device-side position advance and top-k.
 */
#include <float.h>
#include <math.h>

#include "fl_decode.h"
#include "fl_device.cuh"
#include "fl_kernels.h"

namespace {

__device__ __forceinline__ float dq_half(const uint8_t* p) { return __half2float(__ushort_as_half((uint16_t)(p[0] | (p[1] << 8)))); }

/* Dequantizer.cs element formulas with the reference's rounding order
 * (explicit _rn intrinsics: no contraction into FMA). */
__device__ __forceinline__ float dequant_elem(int type, const uint8_t* __restrict__ raw, int64_t f)
{
    switch (type) {
    case FL_T_F32: return __uint_as_float((uint32_t)raw[4 * f] | ((uint32_t)raw[4 * f + 1] << 8) |
                                          ((uint32_t)raw[4 * f + 2] << 16) | ((uint32_t)raw[4 * f + 3] << 24));
    case FL_T_F16: return dq_half(raw + 2 * f);
    case FL_T_BF16: return __uint_as_float(((uint32_t)raw[2 * f] | ((uint32_t)raw[2 * f + 1] << 8)) << 16);
    case FL_T_Q4_0: { /* :178-183 */
        const uint8_t* b = raw + (f / 32) * 18;
        int j = (int)(f % 32);
        int q = j < 16 ? (b[2 + j] & 0x0F) : (b[2 + j - 16] >> 4);
        return __fmul_rn((float)(q - 8), dq_half(b));
    }
    case FL_T_Q8_0: { /* :226-229 */
        const uint8_t* b = raw + (f / 32) * 34;
        return __fmul_rn((float)(int8_t)b[2 + f % 32], dq_half(b));
    }
    case FL_T_Q4_K:
    case FL_T_Q5_K: { /* :268-293, :333-367 */
        const int bb = type == FL_T_Q4_K ? 144 : 176;
        const uint8_t* b = raw + (f / 256) * bb;
        int e = (int)(f % 256);
        int sc, mn;
        fl_kscale_min(b + 4, e / 32, &sc, &mn);
        float dg = __fmul_rn(dq_half(b), (float)sc);
        float mg = __fmul_rn(dq_half(b + 2), (float)mn);
        int q;
        if (type == FL_T_Q4_K) {
            q = (b[16 + (e >> 1)] >> ((e & 1) * 4)) & 0xF;
        } else {
            int lo = (b[48 + (e >> 1)] >> ((e & 1) * 4)) & 0xF;
            int hi = (b[16 + (e >> 3)] >> (e & 7)) & 1;
            q = (hi << 4) | lo;
        }
        return __fsub_rn(__fmul_rn(dg, (float)q), mg);
    }
    case FL_T_Q6_K: { /* :395-416 */
        const uint8_t* b = raw + (f / 256) * 210;
        int i = (int)(f % 256);
        int lo = (b[i >> 1] >> ((i & 1) * 4)) & 0xF;
        int hi = (b[128 + (i >> 2)] >> ((i & 3) * 2)) & 3;
        int q = ((hi << 4) | lo) - 32;
        int s = (int8_t)b[192 + (i >> 4)];
        return __fmul_rn(__fmul_rn(dq_half(b + 208), (float)s), (float)q);
    }
    default: { /* FL_T_Q8_K :444-455 */
        const uint8_t* b = raw + (f / 256) * 292;
        float d = __uint_as_float((uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24));
        return __fmul_rn((float)(int8_t)b[4 + f % 256], d);
    }
    }
}

__global__ void fl_dequant_kernel(int type, const uint8_t* __restrict__ src, int64_t n, float* __restrict__ dst)
{
    for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < n; f += (int64_t)gridDim.x * blockDim.x)
        dst[f] = dequant_elem(type, src, f);
}

/* `_weights.TokenEmbedding.AsSpan(tokenId * h, h).CopyTo(_x)`
 * (LlamaForwardPass.cs:96) over the quantized table: the row is dequantized
 * with the reference formulas, so x matches the reference bit for bit. */
__global__ void fl_embed_kernel(const __grid_constant__ FlEmbedArgs a)
{
    fl_pdl_trigger();
    fl_pdl_wait();
    int tok = *a.token;
    if (tok < 0 || tok >= a.vocab) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(a.err, FL_DEV_ERR_TOKEN);
        tok = 0;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.hidden; i += gridDim.x * blockDim.x)
        a.x[i] = dequant_elem(a.ggml_type, a.raw, (int64_t)tok * a.hidden + i);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.zero_n; i += gridDim.x * blockDim.x) a.zero_buf[i] = 0.0f;
}

__global__ void fl_advance_kernel(const __grid_constant__ FlAdvanceArgs a)
{
    fl_pdl_trigger();
    fl_pdl_wait();
    if (threadIdx.x == 0) {
        int id = *a.argmax;
        int s = *a.step;
        if (a.out_tokens) a.out_tokens[s] = id;
        *a.step = s + 1;
        *a.token = id;
        *a.pos = *a.pos + 1;
    }
}

/* ── attention ──────────────────────────────────────────────────────────
 * ComputeAttention (LlamaForwardPass.cs:158-211; MistralForwardPass.cs:186-240;
 * Gemma2ForwardPass.cs:126-185): per query head, scores over the cached keys
 * [max(0, L-window), L) scaled after the dot, optional softcap, softmax and the
 * weighted sum of values.  Grid (kv_head, split): each CTA reads its slice of
 * keys/values once for all query heads of the group and keeps an online
 * softmax; the last CTA of a kv head merges the splits in split order. */
template <int HD, int GRP>
__global__ void __launch_bounds__(128) fl_attn_kernel(const __grid_constant__ FlAttnArgs a)
{
    constexpr int PER = HD / 32;
    const int kvh = blockIdx.x, split = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv_dim = a.n_kv * HD;
    __shared__ float sq[GRP * HD];
    __shared__ float sm[4][GRP][2];
    __shared__ float sacc[4][GRP][HD];
    __shared__ int s_last;
    fl_pdl_trigger();
    fl_pdl_wait();
    const int seq = *a.pos + 1;
    int start = 0;
    if (a.window < seq) start = seq - a.window;
    const int L = seq - start;
    const int per = (L + a.n_split - 1) / a.n_split;
    const int k0 = start + split * per;
    const int k1 = min(seq, k0 + per);
    for (int i = threadIdx.x; i < GRP * HD; i += blockDim.x) sq[i] = a.q[(size_t)kvh * GRP * HD + i];
    __syncthreads();

    float m[GRP], l[GRP], acc[GRP][PER];
#pragma unroll
    for (int h = 0; h < GRP; h++) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
#pragma unroll
        for (int p = 0; p < PER; p++) acc[h][p] = 0.0f;
    }
    const float inv_cap = a.softcap > 0.0f ? 1.0f / a.softcap : 0.0f;
    for (int t = k0 + warp; t < k1; t += 4) {
        const float* kr = a.k_cache + (size_t)t * kv_dim + (size_t)kvh * HD;
        const float* vr = a.v_cache + (size_t)t * kv_dim + (size_t)kvh * HD;
        float kk[PER], vv[PER];
#pragma unroll
        for (int p = 0; p < PER; p++) {
            kk[p] = kr[lane + 32 * p];
            vv[p] = vr[lane + 32 * p];
        }
#pragma unroll
        for (int h = 0; h < GRP; h++) {
            float s = 0.0f;
#pragma unroll
            for (int p = 0; p < PER; p++) s = fmaf(sq[h * HD + lane + 32 * p], kk[p], s);
            s = fl_warp_sum(s);
            s = __fmul_rn(s, a.scale);
            if (a.softcap > 0.0f) s = __fmul_rn(tanhf(__fmul_rn(s, inv_cap)), a.softcap);
            const float mn = fmaxf(m[h], s);
            const float alpha = expf(m[h] - mn);
            const float pr = expf(s - mn);
            l[h] = fmaf(l[h], alpha, pr);
#pragma unroll
            for (int p = 0; p < PER; p++) acc[h][p] = fmaf(acc[h][p], alpha, pr * vv[p]);
            m[h] = mn;
        }
    }
    /* merge the 4 warps of the CTA */
#pragma unroll
    for (int h = 0; h < GRP; h++) {
        if (lane == 0) {
            sm[warp][h][0] = m[h];
            sm[warp][h][1] = l[h];
        }
#pragma unroll
        for (int p = 0; p < PER; p++) sacc[warp][h][lane + 32 * p] = acc[h][p];
    }
    __syncthreads();
    float* part = a.part + ((size_t)kvh * a.n_split + split) * GRP * (HD + 2);
    for (int i = threadIdx.x; i < GRP * HD; i += blockDim.x) {
        const int h = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int w = 0; w < 4; w++) M = fmaxf(M, sm[w][h][0]);
        float Ls = 0.0f, O = 0.0f;
        for (int w = 0; w < 4; w++) {
            float mw = sm[w][h][0];
            float f = mw == -INFINITY ? 0.0f : expf(mw - M);
            Ls = fmaf(sm[w][h][1], f, Ls);
            O = fmaf(sacc[w][h][d], f, O);
        }
        part[h * (HD + 2) + 2 + d] = O;
        if (d == 0) {
            part[h * (HD + 2)] = M;
            part[h * (HD + 2) + 1] = Ls;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&a.counter[kvh], 1) == a.n_split - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    float amax = 0.0f;
    const float* pk = a.part + (size_t)kvh * a.n_split * GRP * (HD + 2);
    for (int i = threadIdx.x; i < GRP * HD; i += blockDim.x) {
        const int h = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int s = 0; s < a.n_split; s++) M = fmaxf(M, __ldcg(&pk[((size_t)s * GRP + h) * (HD + 2)]));
        float Ls = 0.0f, O = 0.0f;
        for (int s = 0; s < a.n_split; s++) {
            const float* ps = pk + ((size_t)s * GRP + h) * (HD + 2);
            float ms = __ldcg(&ps[0]);
            float f = ms == -INFINITY ? 0.0f : expf(ms - M);
            Ls = fmaf(__ldcg(&ps[1]), f, Ls);
            O = fmaf(__ldcg(&ps[2 + d]), f, O);
        }
        float o = Ls > 0.0f ? O / Ls : 0.0f;
        a.out[((size_t)kvh * GRP + h) * HD + d] = o;
        amax = fmaxf(amax, fabsf(o));
    }
    amax = fl_warp_max(amax);
    if (lane == 0) atomicMax(reinterpret_cast<int*>(a.out_absmax), __float_as_int(amax));
    if (threadIdx.x == 0) a.counter[kvh] = 0;
}

template <int HD, int GRP>
cudaError_t launch_attn(const FlAttnArgs& a, cudaStream_t st, bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.n_kv, (unsigned)a.n_split);
    cfg.blockDim = dim3(128);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fl_attn_kernel<HD, GRP>, a);
}

template <int HD>
cudaError_t launch_attn_hd(const FlAttnArgs& a, cudaStream_t st, bool pdl)
{
    switch (a.n_heads / a.n_kv) {
    case 1: return launch_attn<HD, 1>(a, st, pdl);
    case 2: return launch_attn<HD, 2>(a, st, pdl);
    case 4: return launch_attn<HD, 4>(a, st, pdl);
    case 8: return launch_attn<HD, 8>(a, st, pdl);
    default: return cudaErrorInvalidValue;
    }
}

/* ── top-k ──────────────────────────────────────────────────────────────
 * Radix select of the k-th largest on order-preserving keys, then the
 * (value desc, index asc) order of the k winners. */
__device__ __forceinline__ uint32_t order_key(float f)
{
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void fl_topk_kernel(const float* __restrict__ x, int n, int k, int* __restrict__ ids,
                               float* __restrict__ vals, uint32_t* __restrict__ cand_key, int* __restrict__ cand_idx,
                               int cand_cap)
{
    /* single CTA of 1024 threads */
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_k, s_cnt;
    if (threadIdx.x == 0) {
        s_prefix = 0;
        s_mask = 0;
        s_k = k;
        s_cnt = 0;
    }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            uint32_t key = order_key(x[i]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFF], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int need = s_k;
            int b = 255;
            for (; b > 0; b--) {
                if ((int)hist[b] >= need) break;
                need -= (int)hist[b];
            }
            s_k = need;
            s_prefix = prefix | ((uint32_t)b << shift);
            s_mask = mask | (0xFFu << shift);
        }
        __syncthreads();
    }
    const uint32_t thr = s_prefix; /* key of the k-th largest */
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        uint32_t key = order_key(x[i]);
        if (key >= thr) {
            int p = atomicAdd(&s_cnt, 1);
            if (p < cand_cap) {
                cand_key[p] = key;
                cand_idx[p] = i;
            }
        }
    }
    __syncthreads();
    const int m = min(s_cnt, cand_cap);
    /* rank each candidate: larger key first, then lower index */
    for (int c = threadIdx.x; c < m; c += blockDim.x) {
        uint32_t kc = cand_key[c];
        int ic = cand_idx[c];
        int rank = 0;
        for (int o = 0; o < m; o++) {
            uint32_t ko = cand_key[o];
            int io = cand_idx[o];
            rank += (ko > kc) || (ko == kc && io < ic);
        }
        if (rank < k) {
            ids[rank] = ic;
            vals[rank] = x[ic];
        }
    }
}

} // namespace

cudaError_t fl_launch_dequant(int32_t type, const uint8_t* src, int64_t n, float* dst, cudaStream_t st)
{
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    if (blocks < 1) blocks = 1;
    fl_dequant_kernel<<<(unsigned)blocks, 256, 0, st>>>(type, src, n, dst);
    return cudaGetLastError();
}

cudaError_t fl_launch_embed(const FlEmbedArgs& a, cudaStream_t st, bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.hidden + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fl_embed_kernel, a);
}

cudaError_t fl_launch_advance(const FlAdvanceArgs& a, cudaStream_t st, bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fl_advance_kernel, a);
}

cudaError_t fl_launch_attention(const FlAttnArgs& a, cudaStream_t st, bool pdl)
{
    switch (a.head_dim) {
    case 64: return launch_attn_hd<64>(a, st, pdl);
    case 128: return launch_attn_hd<128>(a, st, pdl);
    case 256: return launch_attn_hd<256>(a, st, pdl);
    default: return cudaErrorInvalidValue;
    }
}

size_t fl_topk_scratch_bytes(int32_t n, int32_t k)
{
    (void)k;
    return (size_t)n * 8;
}

cudaError_t fl_launch_topk(const float* logits, int32_t n, int32_t k, int32_t* ids, float* vals, uint8_t* scratch,
                           size_t scratch_bytes, cudaStream_t st)
{
    int cap = (int)(scratch_bytes / 8);
    uint32_t* ck = reinterpret_cast<uint32_t*>(scratch);
    int* ci = reinterpret_cast<int*>(scratch + (size_t)cap * 4);
    fl_topk_kernel<<<1, 1024, 0, st>>>(logits, n, k, ids, vals, ck, ci, cap);
    return cudaGetLastError();
}
