/*
 * fl_prefill.cu — the prompt path: all prompt tokens of a chunk through one
 * layer at a time (the reference feeds them one by one, LlamaLanguageModel.cs:
 * 133-137; the values are those of LlamaForwardPass.Forward for each token).
 *
 * The projections are dense contractions of the chunk's [n x K] activations
 * with the layer's weights, on the tcgen05 tensor cores (fl_tc_gemm.cu) in
 * split fp16 ("fp16x3"): every operand value v is stored as hi = fp16(v) and
 * lo = fp16(v - hi), and one GEMM over K' = 3K with rows [x_lo | x_hi | x_hi]
 * and [w_hi | w_lo | w_hi] sums x_lo*w_hi + x_hi*w_lo + x_hi*w_hi in fp32 —
 * close to fp32 products of the bit-exact dequantized weights (weights are
 * scaled by FL_PF_WSCALE first so their lo parts stay normal fp16).  The two
 * small cross terms come first: the tensor cores' fp32 accumulation keeps
 * fewer bits of a term added to a larger running sum, so adding them before
 * the hi*hi products, while the sum is small, keeps their bits (measured: 4x
 * less error over K = 14336 than hi*hi first).  A value whose hi part
 * overflows fp16 (|weight| > 65504 / FL_PF_WSCALE, |activation| > 65504) is
 * reported (FL_DEV_ERR_RANGE) instead of stored as infinity.  These kernels do
 * the rest:
 * embedding rows, the residual adds fused with the norms, bias + RoPE + K/V
 * append, causal attention over the KV cache, and the gated FFN activation.
 */
#include <cuda_fp16.h>
#include <math.h>

#include "fl_dequant.cuh"
#include "fl_device.cuh"
#include "fl_kernels.h"

namespace {

/* silu / gelu with the reference's evaluation order (TensorOperations.cs:78-87,
 * 110-117), as in the decode epilogue */
__device__ __forceinline__ float pf_silu(float g)
{
    float sig = 1.0f / __fadd_rn(1.0f, expf(-g));
    return __fmul_rn(g, sig);
}

__device__ __forceinline__ float pf_gelu(float v)
{
    float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
    float inner = __fmul_rn(0.7978845608f, __fadd_rn(v, cube));
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
}

/* A finite value whose fp16 hi part overflowed: recorded once (an earlier
 * error of the launch is kept). */
__device__ __forceinline__ void check_range(__half hi, float v, int* err)
{
    if (err && __hisinf(hi) && isfinite(v)) atomicCAS(err, 0, FL_DEV_ERR_RANGE);
}

/* v into the split layout of its row: [lo | hi | hi] (activations) or
 * [hi | lo | hi] (weights), K values per part */
__device__ __forceinline__ void store_split(__half* row3, int K, int c, float v, bool weight, int* err)
{
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(v - __half2float(hi));
    check_range(hi, v, err);
    row3[c] = weight ? hi : lo;
    row3[K + c] = weight ? lo : hi;
    row3[2 * K + c] = hi;
}

/* An activation value of row r, column c (K per row): the split layout
 * [lo | hi | hi] (rows of 3K) when stack == 0; else stacked for the batched
 * steps' GEMM (rows of 2K): [hi | hi] in row r, [0 | lo] in row stack + r. */
__device__ __forceinline__ void store_act(__half* out, int K, int r, int c, float v, int stack, int* err)
{
    if (stack == 0) {
        store_split(out + (size_t)r * 3 * K, K, c, v, false, err);
        return;
    }
    const __half hi = __float2half_rn(v);
    check_range(hi, v, err);
    __half* rh = out + (size_t)r * 2 * K;
    __half* rl = out + (size_t)(stack + r) * 2 * K;
    rh[c] = hi;
    rh[K + c] = hi;
    rl[c] = __float2half_rn(0.0f);
    rl[K + c] = __float2half_rn(v - __half2float(hi));
}

/* A weight value: [hi | lo | hi] rows of 3K (layout 0) or [lo | hi] rows of 2K (layout 1). */
__device__ __forceinline__ void store_weight(__half* dst, int64_t r, int K, int c, float v, int layout, int* err)
{
    if (layout == 0) {
        store_split(dst + r * 3 * K, K, c, v, true, err);
        return;
    }
    const __half hi = __float2half_rn(v);
    check_range(hi, v, err);
    dst[r * 2 * K + c] = __float2half_rn(v - __half2float(hi));
    dst[r * 2 * K + K + c] = hi;
}

__global__ void dequant_split_kernel(int type, const uint8_t* __restrict__ raw, int64_t n, int cols,
                                     __half* __restrict__ dst, int layout, int* err)
{
    for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < n; f += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = f / cols;
        const int c = (int)(f - r * cols);
        store_weight(dst, r, cols, c, fl_dequant_elem(type, raw, f) * FL_PF_WSCALE, layout, err);
    }
}

/* The 8 consecutive values f0..f0+7 (f0 a multiple of 8) of a quantized
 * matrix: the formulas of fl_dequant_elem, with the block header decoded once
 * and the packed quants read as whole bytes. */
template <int TYPE>
__device__ __forceinline__ void dequant8(const uint8_t* __restrict__ raw, int64_t f0, float (&v)[8])
{
    if constexpr (TYPE == FL_T_Q4_K || TYPE == FL_T_Q5_K) {
        constexpr int bb = TYPE == FL_T_Q4_K ? 144 : 176;
        const uint8_t* b = raw + (f0 / 256) * bb;
        const int e0 = (int)(f0 % 256);
        int sc, mn;
        fl_kscale_min(b + 4, e0 / 32, &sc, &mn);
        const float dg = __fmul_rn(fl_dq_half(b), (float)sc);
        const float mg = __fmul_rn(fl_dq_half(b + 2), (float)mn);
        const uint8_t* qs = b + (TYPE == FL_T_Q4_K ? 16 : 48) + (e0 >> 1);
        const int hb = TYPE == FL_T_Q5_K ? b[16 + (e0 >> 3)] : 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int q = (qs[i >> 1] >> ((i & 1) * 4)) & 0xF;
            if constexpr (TYPE == FL_T_Q5_K) q |= ((hb >> i) & 1) << 4;
            v[i] = __fsub_rn(__fmul_rn(dg, (float)q), mg);
        }
    } else if constexpr (TYPE == FL_T_Q6_K) {
        const uint8_t* b = raw + (f0 / 256) * 210;
        const int i0 = (int)(f0 % 256);
        const float ds = __fmul_rn(fl_dq_half(b + 208), (float)(int8_t)b[192 + (i0 >> 4)]);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int e = i0 + i;
            const int lo = (b[e >> 1] >> ((e & 1) * 4)) & 0xF;
            const int hi = (b[128 + (e >> 2)] >> ((e & 3) * 2)) & 3;
            v[i] = __fmul_rn(ds, (float)(((hi << 4) | lo) - 32));
        }
    } else if constexpr (TYPE == FL_T_Q8_0) {
        const uint8_t* b = raw + (f0 / 32) * 34;
        const int j0 = (int)(f0 % 32);
        const float d = fl_dq_half(b);
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = __fmul_rn((float)(int8_t)b[2 + j0 + i], d);
    } else { /* Q4_0 */
        const uint8_t* b = raw + (f0 / 32) * 18;
        const int j0 = (int)(f0 % 32);
        const float d = fl_dq_half(b);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int j = j0 + i;
            const int q = j < 16 ? (b[2 + j] & 0x0F) : (b[2 + j - 16] >> 4);
            v[i] = __fmul_rn((float)(q - 8), d);
        }
    }
}

/* Weights in the split layout [hi | lo | hi] (scaled by FL_PF_WSCALE), 8
 * values per thread, each part written as one 16-byte store. */
template <int TYPE>
__global__ void dequant_split8_kernel(const uint8_t* __restrict__ raw, int64_t n8, int cols, __half* __restrict__ dst,
                                      int layout, int* err)
{
    for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < n8; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t f0 = g * 8;
        float v[8];
        dequant8<TYPE>(raw, f0, v);
        const int64_t r = f0 / cols;
        const int c = (int)(f0 - r * cols);
        __align__(16) __half hi[8], lo[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float x = v[i] * FL_PF_WSCALE;
            hi[i] = __float2half_rn(x);
            lo[i] = __float2half_rn(x - __half2float(hi[i]));
            check_range(hi[i], x, err);
        }
        const uint4 h4 = *reinterpret_cast<const uint4*>(hi), l4 = *reinterpret_cast<const uint4*>(lo);
        if (layout == 0) {
            __half* row3 = dst + r * 3 * (int64_t)cols;
            *reinterpret_cast<uint4*>(row3 + c) = h4;
            *reinterpret_cast<uint4*>(row3 + cols + c) = l4;
            *reinterpret_cast<uint4*>(row3 + 2 * cols + c) = h4;
        } else {
            __half* row2 = dst + r * 2 * (int64_t)cols;
            *reinterpret_cast<uint4*>(row2 + c) = l4;
            *reinterpret_cast<uint4*>(row2 + cols + c) = h4;
        }
    }
}

__global__ void embed_rows_kernel(int type, const uint8_t* __restrict__ raw, const int32_t* __restrict__ tokens,
                                  int h, int vocab, float* __restrict__ x, int* err)
{
    const int r = blockIdx.x;
    int tok = tokens[r];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicExch(err, FL_DEV_ERR_TOKEN);
        tok = 0;
    }
    for (int i = threadIdx.x; i < h; i += blockDim.x)
        x[(size_t)r * h + i] = fl_dequant_elem(type, raw, (int64_t)tok * h + i);
}

__device__ float block_sum(float v, float* red)
{
    v = fl_warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
    return t;
}

/* One row per CTA: optionally x += y (Gemma: x += GemmaRmsNorm(y, post_w)),
 * then out = norm(x) * w as fp16 (RmsNorm, or GemmaRmsNorm with w + 1). */
__global__ void rows_norm_kernel(float* __restrict__ x, const float* __restrict__ y, const float* __restrict__ post_w,
                                 const float* __restrict__ w, int h, float eps, int gemma, __half* __restrict__ out,
                                 int stack, const float* __restrict__ y_lo, int* err)
{
    /* y_lo (the two-GEMM form's second half, or NULL) is part of y */
    __shared__ float red[32];
    const int r = blockIdx.x;
    float* xr = x + (size_t)r * h;
    if (y) {
        const float* yr = y + (size_t)r * h;
        const float* yl = y_lo ? y_lo + (size_t)r * h : nullptr;
        auto yv = [&](int i) { return yl ? __fadd_rn(yr[i], yl[i]) : yr[i]; };
        float rp = 1.0f;
        if (post_w) {
            float sp = 0.0f;
            for (int i = threadIdx.x; i < h; i += blockDim.x) {
                const float v = yv(i);
                sp = fmaf(v, v, sp);
            }
            sp = block_sum(sp, red);
            rp = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(sp, (float)h), 1e-6f));
        }
        for (int i = threadIdx.x; i < h; i += blockDim.x) {
            const float add = post_w ? __fmul_rn(__fmul_rn(yv(i), rp), __fadd_rn(post_w[i], 1.0f)) : yv(i);
            xr[i] = __fadd_rn(xr[i], add);
        }
        __syncthreads();
    }
    if (!out) return;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < h; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = block_sum(ss, red);
    const float rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)h), eps));
    for (int i = threadIdx.x; i < h; i += blockDim.x) {
        const float wi = gemma ? __fadd_rn(w[i], 1.0f) : w[i];
        store_act(out, h, r, i, __fmul_rn(__fmul_rn(xr[i], rms), wi), stack, err);
    }
}

/* q, k, v of token r (GEMM output row [q | k | v]): bias, RoPE on q and k
 * (TensorOperations.ApplyRope, the decode epilogue's order), q to q_out,
 * k and v into the cache at position start_pos + r. */
__global__ void rope_kv_kernel(const float* __restrict__ qkv, const float* __restrict__ bq, const float* __restrict__ bk,
                               const float* __restrict__ bv, const float* __restrict__ rope_cs, int start_pos, int qd,
                               int kvd, int hd, float* __restrict__ q_out, float* __restrict__ k_cache,
                               float* __restrict__ v_cache, const int* __restrict__ row_pos,
                               const int* __restrict__ row_slot, size_t slot_stride, const float* __restrict__ qkv_lo)
{
    /* row r is position start_pos + r of one sequence, or (batched decode)
     * position row_pos[r] of the sequence in cache slot row_slot[r] */
    const int r = blockIdx.x, pos = row_pos ? row_pos[r] : start_pos + r, half = hd >> 1;
    if (row_slot) {
        k_cache += (size_t)row_slot[r] * slot_stride;
        v_cache += (size_t)row_slot[r] * slot_stride;
    }
    const int width = qd + 2 * kvd;
    const float* row = qkv + (size_t)r * width;
    const float* row_lo = qkv_lo ? qkv_lo + (size_t)r * width : nullptr; /* the second half, or NULL */
    auto at = [&](int j) { return row_lo ? __fadd_rn(row[j], row_lo[j]) : row[j]; };
    for (int j = threadIdx.x; j < width; j += blockDim.x) {
        if (j < qd + kvd) {
            const bool is_q = j < qd;
            const int e = is_q ? j : j - qd;
            const float* b = is_q ? bq : bk;
            const int pe = e ^ 1;
            float v = at(j), partner = at(is_q ? pe : qd + pe);
            if (b) {
                v = __fadd_rn(v, b[e]);
                partner = __fadd_rn(partner, b[pe]);
            }
            const int d = e % hd, i = d >> 1;
            const float2 cs = *reinterpret_cast<const float2*>(rope_cs + ((size_t)pos * half + i) * 2);
            float o;
            if ((d & 1) == 0) o = __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(partner, cs.y));
            else o = __fadd_rn(__fmul_rn(partner, cs.y), __fmul_rn(v, cs.x));
            if (is_q) q_out[(size_t)r * qd + e] = o;
            else k_cache[(size_t)pos * kvd + e] = o;
        } else {
            const int e = j - qd - kvd;
            float v = at(j);
            if (bv) v = __fadd_rn(v, bv[e]);
            v_cache[(size_t)pos * kvd + e] = v;
        }
    }
}

/* ── batched decode: one query per row, each row its own sequence ──────────
 * ComputeAttention (LlamaForwardPass.cs:158-211, windows and softcap as in the
 * Mistral/Gemma passes) for row b, kv head g: the grp query heads of the
 * group against keys [max(0, p+1-window), p+1) of the row's cache slot.  Each
 * of the 8 warps takes KPW = 1024/head_dim keys per round (head_dim/32 lanes
 * per key for the scores, then every lane owns head_dim/32 dims of the
 * values; the round's key and value loads are issued together) and keeps a
 * running (max, sum, output) per head, updated once per round; the warps are
 * merged in warp order. */
template <int HD>
__global__ void __launch_bounds__(256) batch_attn_kernel(const float* __restrict__ q, const float* __restrict__ k_cache,
                                                        const float* __restrict__ v_cache,
                                                        const int* __restrict__ row_pos,
                                                        const int* __restrict__ row_slot, size_t slot_stride, int nh,
                                                        int nkv, int window, float scale, float softcap,
                                                        __half* __restrict__ out, int stack, int* err)
{
    constexpr int GM = HD == 256 ? 4 : 8, NWB = 8; /* GM: largest query-head group */
    constexpr int LPK = HD / 32, KPW = 32 / LPK, PER = HD / 32;
    __shared__ __align__(16) float sq[GM][HD];
    __shared__ float s_o[NWB][GM][HD];
    __shared__ float s_ml[NWB][GM][2];
    const int b = blockIdx.x, g = blockIdx.y, grp = nh / nkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd4 = lane % LPK, kj = lane / LPK;
    const int qd = nh * HD, kvd = nkv * HD;
    const int pos = row_pos[b];
    const int k_lo = window < pos + 1 ? pos + 1 - window : 0;
    const int n = pos + 1 - k_lo;
    const float* kc = k_cache + (size_t)row_slot[b] * slot_stride + (size_t)k_lo * kvd + (size_t)g * HD;
    const float* vc = v_cache + (size_t)row_slot[b] * slot_stride + (size_t)k_lo * kvd + (size_t)g * HD + lane * PER;
    const float inv_cap = softcap > 0.0f ? 1.0f / softcap : 0.0f;
    for (int i = threadIdx.x; i < grp * HD; i += blockDim.x) sq[i / HD][i % HD] = q[(size_t)b * qd + (size_t)g * grp * HD + i];
    __syncthreads();
    float m[GM], l[GM], o[GM][PER];
#pragma unroll
    for (int h = 0; h < GM; h++) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
#pragma unroll
        for (int p = 0; p < PER; p++) o[h][p] = 0.0f;
    }
    for (int base = warp * KPW; base < n; base += NWB * KPW) {
        const bool valid = base + kj < n;
        float4 kv[8];
        float vv[KPW][PER];
        const int kk = min(base + kj, n - 1);
#pragma unroll
        for (int c = 0; c < 8; c++) kv[c] = *(reinterpret_cast<const float4*>(kc + (size_t)kk * kvd) + c * LPK + qd4);
#pragma unroll
        for (int j = 0; j < KPW; j++) {
            const int t = min(base + j, n - 1);
#pragma unroll
            for (int p = 0; p < PER; p++) vv[j][p] = vc[(size_t)t * kvd + p];
        }
#pragma unroll
        for (int h = 0; h < GM; h++) {
            if (h >= grp) break;
            float acc = 0.0f;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const float4 q4 = reinterpret_cast<const float4*>(sq[h])[c * LPK + qd4];
                acc = fmaf(q4.x, kv[c].x, acc);
                acc = fmaf(q4.y, kv[c].y, acc);
                acc = fmaf(q4.z, kv[c].z, acc);
                acc = fmaf(q4.w, kv[c].w, acc);
            }
#pragma unroll
            for (int off = 1; off < LPK; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
            float sc = __fmul_rn(acc, scale);
            if (softcap > 0.0f) sc = __fmul_rn(tanhf(__fmul_rn(sc, inv_cap)), softcap);
            sc = valid ? sc : -INFINITY;
            float mr = sc; /* the round's max (key `base` is valid) */
#pragma unroll
            for (int off = LPK; off < 32; off <<= 1) mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, off));
            const float mn = fmaxf(m[h], mr);
            const float corr = __expf(m[h] - mn); /* 0 on the first round */
            const float pw = __expf(sc - mn);     /* 0 past the keys */
            m[h] = mn;
            l[h] *= corr;
#pragma unroll
            for (int p = 0; p < PER; p++) o[h][p] *= corr;
#pragma unroll
            for (int j = 0; j < KPW; j++) {
                const float pj = __shfl_sync(0xffffffffu, pw, j * LPK);
                l[h] += pj;
#pragma unroll
                for (int p = 0; p < PER; p++) o[h][p] = fmaf(pj, vv[j][p], o[h][p]);
            }
        }
    }
#pragma unroll
    for (int h = 0; h < GM; h++) {
        if (h >= grp) break;
#pragma unroll
        for (int p = 0; p < PER; p++) s_o[warp][h][lane * PER + p] = o[h][p];
        if (lane == 0) {
            s_ml[warp][h][0] = m[h];
            s_ml[warp][h][1] = l[h];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < grp * HD; i += blockDim.x) {
        const int h = i / HD, d = i - h * HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NWB; w++) M = fmaxf(M, s_ml[w][h][0]);
        float O = 0.0f, L = 0.0f;
#pragma unroll
        for (int w = 0; w < NWB; w++) {
            const float mw = s_ml[w][h][0];
            const float f = mw == -INFINITY ? 0.0f : __expf(mw - M);
            O = fmaf(s_o[w][h][d], f, O);
            L = fmaf(s_ml[w][h][1], f, L);
        }
        store_act(out, qd, b, (g * grp + h) * HD + d, L > 0.0f ? O / L : 0.0f, stack, err);
    }
}

/* The two-GEMM form's halves: y[b][j] = p[b][j] + p[B + b][j]. */
__global__ void add_halves_kernel(const float* __restrict__ p, int B, int N, float* __restrict__ y)
{
    const size_t total = (size_t)B * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(p[i], p[total + i]);
}

/* TensorOperations.SoftCap (TensorOperations.cs:120-126) on logits rows */
__global__ void softcap_kernel(float* __restrict__ x, size_t n, float cap)
{
    const float inv = 1.0f / cap;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        x[i] = __fmul_rn(tanhf(__fmul_rn(x[i], inv)), cap);
}

/* TensorOperations.ArgMax per row (the first maximum). */
__global__ void argmax_rows_kernel(const float* __restrict__ x, int n, int* __restrict__ out)
{
    __shared__ float sv[16];
    __shared__ int si[16];
    const float* row = x + (size_t)blockIdx.x * n;
    float bv = 0.0f;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = row[i];
        if (bi == 0x7fffffff || fl_argmax_better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oi != 0x7fffffff && (bi == 0x7fffffff || fl_argmax_better(ov, oi, bv, bi))) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = sv[0];
        int i0 = si[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (si[w] != 0x7fffffff && (i0 == 0x7fffffff || fl_argmax_better(sv[w], si[w], v, i0))) {
                v = sv[w];
                i0 = si[w];
            }
        out[blockIdx.x] = i0;
    }
}

/* ── tensor parallelism: the allreduce of a chunk's row-parallel partials ── */

/* This rank's partial slot is complete (the GEMM before this launch wrote it):
 * publish it to every rank by raising this rank's flag there to `epoch`. */
struct TpFlags {
    int* f[FL_TP_MAX]; /* every rank's flag array (passed by value) */
};

__global__ void tp_pf_signal_kernel(TpFlags flags, int T, int rank, int epoch)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    __threadfence_system();
    for (int q = 0; q < T; q++) fl_st_release_sys(flags.f[q] + rank, epoch);
}

struct TpSlots {
    const float* slot[FL_TP_MAX];
    const int* my_flags; /* this rank's flag array, which the peers write */
};

/* Waits (bounded, ~2 s) for every rank's flag to reach `epoch`, then sums the
 * T partial slots in rank order (peers over NVLink) into y. */
__global__ void tp_pf_reduce_kernel(TpSlots sl, int T, int epoch, size_t count, float* __restrict__ y, int* err)
{
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        int ok = !fl_err_set(err); /* an earlier exchange of this prompt already gave up */
        const uint64_t t0 = fl_globaltimer();
        for (int q = 0; q < T && ok; q++)
            for (uint32_t it = 0; fl_ld_acquire_sys(sl.my_flags + q) < epoch; it++)
                if ((it & 255u) == 0 && (fl_err_set(err) || fl_globaltimer() - t0 > 2000000000ull)) {
                    if (!fl_err_set(err)) atomicExch(err, FL_DEV_ERR_TIMEOUT);
                    ok = 0;
                    break;
                }
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
        float sum = 0.0f;
        for (int q = 0; q < T; q++) sum += fl_ld_relaxed_sys(sl.slot[q] + i);
        y[i] = sum;
    }
}

/* ── causal attention of a chunk on the tensor cores ────────────────────────
 * Per kv head g (a GEMM batch), the chunk's queries of all grp query heads of
 * the group are the rows (t, h) = t*grp + h of one matrix, so one split-fp16
 * GEMM forms every score against the keys 0..nk of the cache (earlier chunks
 * included); a row kernel applies the scale, softcap, causal and window masks
 * and the softmax; a second split-fp16 GEMM multiplies the probabilities
 * (times 2^10, so their lo parts stay normal) by the values. */

/* Q rows into [lo | hi | hi] per head, grouped by kv head. */
__global__ void attn_q_split_kernel(const float* __restrict__ q, int n, int nh, int nkv, int hd, __half* __restrict__ qs,
                                    int* err)
{
    const int t = blockIdx.x, qd = nh * hd, grp = nh / nkv;
    for (int i = threadIdx.x; i < qd; i += blockDim.x) {
        const int head = i / hd, d = i - head * hd, g = head / grp, h = head - g * grp;
        __half* row = qs + ((size_t)g * n * grp + (size_t)t * grp + h) * 3 * hd;
        store_split(row, hd, d, q[(size_t)t * qd + i], false, err);
    }
}

/* Keys 0..nkp of every kv head into [hi | lo | hi] rows; values transposed,
 * one [hi | lo | hi] row of nkp keys per (kv head, dim); zero past nk.  A
 * 32-key x 32-dim tile per block, staged so both sides are coalesced. */
__global__ void attn_kv_split_kernel(const float* __restrict__ kc, const float* __restrict__ vc, int nk, int nkp,
                                     int kvd, int hd, __half* __restrict__ ks, __half* __restrict__ vt, int* err)
{
    __shared__ float tile[32][33];
    const int k0 = blockIdx.x * 32, c0 = blockIdx.y * 32, tx = threadIdx.x, ty = threadIdx.y;
    for (int r = ty; r < 32; r += 8) {
        const int key = k0 + r, c = c0 + tx;
        const bool ok = key < nk && c < kvd;
        const float kv = ok ? kc[(size_t)key * kvd + c] : 0.0f;
        const float vv = ok ? vc[(size_t)key * kvd + c] : 0.0f;
        if (key < nkp && c < kvd) {
            const int g = c / hd, d = c - g * hd;
            store_split(ks + ((size_t)g * nkp + key) * 3 * hd, hd, d, kv, true, err);
        }
        tile[r][tx] = vv;
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
        const int c = c0 + r, key = k0 + tx;
        if (c < kvd && key < nkp) {
            const int g = c / hd, d = c - g * hd;
            store_split(vt + ((size_t)g * hd + d) * 3 * nkp, nkp, key, tile[tx][r], true, err);
        }
    }
}

__device__ float attn_block_reduce(float v, bool is_max, float* red)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = is_max ? fl_warp_max(v) : fl_warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < (int)(blockDim.x >> 5) ? red[lane] : (is_max ? -INFINITY : 0.0f);
        t = is_max ? fl_warp_max(t) : fl_warp_sum(t);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

/* Row (g, t, h): ComputeAttention's score (dot * scale [→ softcap]) over the
 * keys [max(0, p+1-window), p+1) of position p = start + t, then Softmax
 * (max, exp(s - max), sum, divide); written as 2^10 * p in [lo | hi | hi]. */
template <bool STAGED>
__global__ void attn_softmax_kernel(const float* __restrict__ S, int n, int grp, int nkp, int start, int window,
                                    float scale, float softcap, __half* __restrict__ P)
{
    __shared__ float red[33];
    extern __shared__ float srow_s[]; /* STAGED: the row's scores, then exp(score - max) */
    const size_t row = blockIdx.x;
    const int t = (int)((row % ((size_t)n * grp)) / grp), pos = start + t;
    const int k_lo = window < pos + 1 ? pos + 1 - window : 0, k_hi = pos;
    const float* srow = S + row * nkp;
    __half* prow = P + row * 3 * (size_t)nkp;
    const float inv_cap = softcap > 0.0f ? 1.0f / softcap : 0.0f;
    auto score = [&](int k) {
        float v = __fmul_rn(srow[k], scale);
        if (softcap > 0.0f) v = __fmul_rn(tanhf(__fmul_rn(v, inv_cap)), softcap);
        return v;
    };
    float mx = -INFINITY;
    for (int k = k_lo + threadIdx.x; k <= k_hi; k += blockDim.x) {
        const float v = score(k);
        if constexpr (STAGED) srow_s[k] = v;
        mx = fmaxf(mx, v);
    }
    mx = attn_block_reduce(mx, true, red);
    float sum = 0.0f;
    for (int k = k_lo + threadIdx.x; k <= k_hi; k += blockDim.x) {
        const float e = expf(__fsub_rn(STAGED ? srow_s[k] : score(k), mx));
        if constexpr (STAGED) srow_s[k] = e;
        sum += e;
    }
    sum = attn_block_reduce(sum, false, red);
    for (int k = threadIdx.x; k < nkp; k += blockDim.x) {
        float p = 0.0f;
        if (k >= k_lo && k <= k_hi) p = __fdiv_rn(STAGED ? srow_s[k] : expf(__fsub_rn(score(k), mx)), sum);
        store_split(prow, nkp, k, p * 1024.0f, false, nullptr); /* |2^10 p| <= 1024 */
    }
}

/* The attention output rows (g, t, h) into the Wo input layout [t][qd]. */
__global__ void attn_out_kernel(const float* __restrict__ O, int n, int nh, int nkv, int hd, __half* __restrict__ act,
                                int* err)
{
    const int t = blockIdx.x, qd = nh * hd, grp = nh / nkv;
    for (int i = threadIdx.x; i < qd; i += blockDim.x) {
        const int head = i / hd, d = i - head * hd, g = head / grp, h = head - g * grp;
        store_split(act + (size_t)t * 3 * qd, qd, i, O[((size_t)g * n * grp + (size_t)t * grp + h) * hd + d], false, err);
    }
}

__global__ void glu_kernel(const float* __restrict__ g, int n, int F, int gelu, __half* __restrict__ act, int stack,
                           const float* __restrict__ g_lo, int* err)
{
    const int64_t total = (int64_t)n * F;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / F, c = i % F;
        float gv = g[r * 2 * F + c], up = g[r * 2 * F + F + c];
        if (g_lo) {
            gv = __fadd_rn(gv, g_lo[r * 2 * F + c]);
            up = __fadd_rn(up, g_lo[r * 2 * F + F + c]);
        }
        store_act(act, F, (int)r, (int)c, __fmul_rn(gelu ? pf_gelu(gv) : pf_silu(gv), up), stack, err);
    }
}

} // namespace

cudaError_t fl_launch_dequant_split(int32_t type, const uint8_t* raw, int rows, int cols, __half* dst, cudaStream_t st,
                                    int layout, int* err)
{
    const int64_t n = (int64_t)rows * cols;
    if (cols % 8 == 0) {
        const int64_t n8 = n / 8;
        int64_t b8 = (n8 + 255) / 256;
        if (b8 > 148 * 16) b8 = 148 * 16;
        if (b8 < 1) b8 = 1;
        switch (type) {
        case FL_T_Q4_K: dequant_split8_kernel<FL_T_Q4_K><<<(unsigned)b8, 256, 0, st>>>(raw, n8, cols, dst, layout, err); return cudaGetLastError();
        case FL_T_Q5_K: dequant_split8_kernel<FL_T_Q5_K><<<(unsigned)b8, 256, 0, st>>>(raw, n8, cols, dst, layout, err); return cudaGetLastError();
        case FL_T_Q6_K: dequant_split8_kernel<FL_T_Q6_K><<<(unsigned)b8, 256, 0, st>>>(raw, n8, cols, dst, layout, err); return cudaGetLastError();
        case FL_T_Q8_0: dequant_split8_kernel<FL_T_Q8_0><<<(unsigned)b8, 256, 0, st>>>(raw, n8, cols, dst, layout, err); return cudaGetLastError();
        case FL_T_Q4_0: dequant_split8_kernel<FL_T_Q4_0><<<(unsigned)b8, 256, 0, st>>>(raw, n8, cols, dst, layout, err); return cudaGetLastError();
        default: break;
        }
    }
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    if (blocks < 1) blocks = 1;
    dequant_split_kernel<<<(unsigned)blocks, 256, 0, st>>>(type, raw, n, cols, dst, layout, err);
    return cudaGetLastError();
}

cudaError_t fl_launch_embed_rows(int32_t type, const uint8_t* raw, const int32_t* tokens, int n, int h, int vocab,
                                 float* x, int* err, cudaStream_t st)
{
    embed_rows_kernel<<<n, 256, 0, st>>>(type, raw, tokens, h, vocab, x, err);
    return cudaGetLastError();
}

cudaError_t fl_launch_rows_norm(float* x, const float* y, const float* post_w, const float* w, int n, int h, float eps,
                                int gemma, __half* out, cudaStream_t st, int stack, const float* y_lo, int* err)
{
    rows_norm_kernel<<<n, n < 148 ? 1024 : 256, 0, st>>>(x, y, post_w, w, h, eps, gemma, out, stack, y_lo, err);
    return cudaGetLastError();
}

cudaError_t fl_launch_rope_kv(const float* qkv, const float* bq, const float* bk, const float* bv, const float* rope_cs,
                              int start_pos, int n, int qd, int kvd, int hd, float* q_out, float* k_cache,
                              float* v_cache, cudaStream_t st)
{
    rope_kv_kernel<<<n, 256, 0, st>>>(qkv, bq, bk, bv, rope_cs, start_pos, qd, kvd, hd, q_out, k_cache, v_cache,
                                      nullptr, nullptr, 0, nullptr);
    return cudaGetLastError();
}

cudaError_t fl_launch_rope_kv_rows(const float* qkv, const float* bq, const float* bk, const float* bv,
                                   const float* rope_cs, const int* row_pos, const int* row_slot, size_t slot_stride,
                                   int n, int qd, int kvd, int hd, float* q_out, float* k_cache, float* v_cache,
                                   cudaStream_t st, const float* qkv_lo)
{
    rope_kv_kernel<<<n, n < 148 ? 1024 : 256, 0, st>>>(qkv, bq, bk, bv, rope_cs, 0, qd, kvd, hd, q_out, k_cache,
                                                       v_cache, row_pos, row_slot, slot_stride, qkv_lo);
    return cudaGetLastError();
}

cudaError_t fl_launch_batch_attn(const float* q, const float* k_cache, const float* v_cache, const int* row_pos,
                                 const int* row_slot, size_t slot_stride, int B, int nh, int nkv, int hd, int window,
                                 float scale, float softcap, __half* out, cudaStream_t st, int stack, int* err)
{
    dim3 grid((unsigned)B, (unsigned)nkv);
    switch (hd) {
    case 64: batch_attn_kernel<64><<<grid, 256, 0, st>>>(q, k_cache, v_cache, row_pos, row_slot, slot_stride, nh, nkv, window, scale, softcap, out, stack, err); break;
    case 128: batch_attn_kernel<128><<<grid, 256, 0, st>>>(q, k_cache, v_cache, row_pos, row_slot, slot_stride, nh, nkv, window, scale, softcap, out, stack, err); break;
    case 256: batch_attn_kernel<256><<<grid, 256, 0, st>>>(q, k_cache, v_cache, row_pos, row_slot, slot_stride, nh, nkv, window, scale, softcap, out, stack, err); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t fl_launch_add_halves(const float* p, int B, int N, float* y, cudaStream_t st)
{
    add_halves_kernel<<<148 * 2, 256, 0, st>>>(p, B, N, y);
    return cudaGetLastError();
}

cudaError_t fl_launch_softcap_rows(float* x, size_t n, float cap, cudaStream_t st)
{
    softcap_kernel<<<148 * 4, 256, 0, st>>>(x, n, cap);
    return cudaGetLastError();
}

cudaError_t fl_launch_argmax_rows(const float* x, int rows, int n, int* out, cudaStream_t st)
{
    argmax_rows_kernel<<<rows, 512, 0, st>>>(x, n, out);
    return cudaGetLastError();
}

cudaError_t fl_launch_tp_prefill_reduce(const float* const* slots, int* const* flags, int T, int rank, int epoch,
                                        size_t count, float* y, int* err, cudaStream_t st)
{
    if (T < 2 || T > FL_TP_MAX || rank < 0 || rank >= T) return cudaErrorInvalidValue;
    TpFlags fl = {};
    TpSlots sl = {};
    for (int q = 0; q < T; q++) {
        fl.f[q] = flags[q];
        sl.slot[q] = slots[q];
    }
    sl.my_flags = flags[rank];
    tp_pf_signal_kernel<<<1, 32, 0, st>>>(fl, T, rank, epoch);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    unsigned blocks = (unsigned)((count + 255) / 256);
    if (blocks > 148) blocks = 148; /* every CTA co-resident: each one waits */
    tp_pf_reduce_kernel<<<blocks, 256, 0, st>>>(sl, T, epoch, count, y, err);
    return cudaGetLastError();
}

cudaError_t fl_launch_attn_q_split(const float* q, int n, int nh, int nkv, int hd, __half* qs, cudaStream_t st, int* err)
{
    attn_q_split_kernel<<<n, 256, 0, st>>>(q, n, nh, nkv, hd, qs, err);
    return cudaGetLastError();
}

cudaError_t fl_launch_attn_kv_split(const float* kc, const float* vc, int nk, int nkp, int kvd, int hd, __half* ks,
                                    __half* vt, cudaStream_t st, int* err)
{
    dim3 grid((unsigned)((nkp + 31) / 32), (unsigned)((kvd + 31) / 32));
    attn_kv_split_kernel<<<grid, dim3(32, 8), 0, st>>>(kc, vc, nk, nkp, kvd, hd, ks, vt, err);
    return cudaGetLastError();
}

cudaError_t fl_launch_attn_softmax(const float* S, int rows, int n, int grp, int nkp, int start, int window, float scale,
                                   float softcap, __half* P, cudaStream_t st)
{
    const size_t smem = (size_t)nkp * 4;
    if (smem <= (size_t)200 * 1024) {
        if (smem > 48 * 1024) {
            const cudaError_t e = cudaFuncSetAttribute(attn_softmax_kernel<true>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
        }
        attn_softmax_kernel<true><<<rows, 256, smem, st>>>(S, n, grp, nkp, start, window, scale, softcap, P);
    } else {
        attn_softmax_kernel<false><<<rows, 256, 0, st>>>(S, n, grp, nkp, start, window, scale, softcap, P);
    }
    return cudaGetLastError();
}

cudaError_t fl_launch_attn_out(const float* O, int n, int nh, int nkv, int hd, __half* act, cudaStream_t st, int* err)
{
    attn_out_kernel<<<n, 256, 0, st>>>(O, n, nh, nkv, hd, act, err);
    return cudaGetLastError();
}

cudaError_t fl_launch_glu(const float* g, int n, int F, int gelu, __half* act, cudaStream_t st, int stack,
                          const float* g_lo, int* err)
{
    const int64_t total = (int64_t)n * F;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    if (blocks < 1) blocks = 1;
    glu_kernel<<<(unsigned)blocks, 256, 0, st>>>(g, n, F, gelu, act, stack, g_lo, err);
    return cudaGetLastError();
}
