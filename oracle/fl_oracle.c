/*
 * fl_oracle.c — CPU restatement of DotNetFoundryLLM v1.0.0's token loop.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker for the CUDA path; see
 * fl_oracle.h).  Built with -ffp-contract=off so that every C# float
 * expression is evaluated with the same number of roundings as RyuJIT emits
 * (RyuJIT never contracts a*b+c into an FMA).
 *
 * Citations are path:line inside the reference repository.
 *
 * Parity notes
 *  - Dequantization (Dequantizer.cs) is restated operation for operation and
 *    is bit-exact: it uses no third-party arithmetic.
 *  - Dot/Softmax/Sigmoid/Exp/Tanh come from System.Numerics.Tensors 10.0.7
 *    (TensorPrimitives, NuGet, not vendored).  Its SIMD reduction order and its
 *    vectorised exp/tanh depend on the host ISA; this file uses an 8-lane
 *    partial-sum dot (the Vector256 shape) and glibc expf/tanhf.  Parity at that
 *    boundary is unpinned and governed by the 1e-2 rel / 1e-3 abs tolerance.
 *  - MathF.Pow/Cos/Sin/Tanh lower to the C runtime (glibc) on Linux; MathF.Sqrt
 *    is the correctly rounded sqrtss.  This file calls the same functions.
 */
#define _GNU_SOURCE
#include "fl_oracle.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <limits.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 1;
void or_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int or_get_threads(void) { return g_threads; }

static void set_err(char* err, int errlen, const char* fmt, ...)
{
    if (!err || errlen <= 0) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, (size_t)errlen, fmt, ap);
    va_end(ap);
}

/* ════════════════════════════════════════════════════════════════════════
 * Quantization/Dequantizer.cs
 * ════════════════════════════════════════════════════════════════════════ */

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const uint8_t* p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static inline uint64_t rd64(const uint8_t* p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }
static inline float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* Dequantizer.HalfToFloat (Dequantizer.cs:50-51): (float)BitConverter.UInt16BitsToHalf.
 * An exact IEEE binary16 → binary32 widening (subnormals, ±inf; NaN payload
 * shifted into the float mantissa). */
float or_half_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t out;
    if (exp == 0) {
        if (man == 0) {
            out = sign;
        } else {
            /* subnormal half: value = man * 2^-24, normalise */
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            out = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1F) {
        /* infinity, or a NaN returned quiet with its payload (the conversion
         * behind (float)Half sets the quiet bit of a signalling NaN) */
        out = man ? (sign | 0x7FC00000u | (man << 13)) : (sign | 0x7F800000u);
    } else {
        out = sign | ((exp + (127 - 15)) << 23) | (man << 13);
    }
    return bits_to_f32(out);
}

/* Dequantizer.BFloat16ToFloat (Dequantizer.cs:58-59): bits << 16. */
float or_bf16_to_float(uint16_t b) { return bits_to_f32((uint32_t)b << 16); }

/* Dequantizer.ElementCount (Dequantizer.cs:466-479). */
int64_t or_element_count(int t, int64_t n)
{
    switch (t) {
    case 0: return n / 4;
    case 1: return n / 2;
    case 2: return n / 18 * 32;
    case 8: return n / 34 * 32;
    case 12: return n / 144 * 256;
    case 13: return n / 176 * 256;
    case 14: return n / 210 * 256;
    case 15: return n / 292 * 256;
    case 30: return n / 2;
    default: return OR_NOT_SUPPORTED;
    }
}

/* DecodeKScaleMin (Dequantizer.cs:506-521). */
static inline void decode_kscale_min(const uint8_t* p, int g, int* sc, int* mn)
{
    if (g < 4) {
        *sc = p[g] & 0x3F;
        *mn = p[g + 4] & 0x3F;
        return;
    }
    int i = g - 4;
    *sc = (p[g + 4] & 0x0F) | ((p[i] >> 6) << 4);
    *mn = (p[g + 4] >> 4) | ((p[i + 4] >> 6) << 4);
}

/* Dequantizer.Dequantize (Dequantizer.cs:488-504) and the per-format methods. */
int or_dequantize(int t, const uint8_t* src, int64_t n, float* dst, int64_t dst_len)
{
    switch (t) {
    case 0: { /* DequantizeF32 :68-85 */
        if (n % 4 != 0) return OR_ARGUMENT_EXCEPTION;
        int64_t c = n / 4;
        if (dst_len < c) return OR_ARGUMENT_EXCEPTION;
        for (int64_t i = 0; i < c; i++) dst[i] = bits_to_f32(rd32(src + 4 * i));
        return OR_OK;
    }
    case 1: { /* DequantizeF16 :94-111 */
        if (n % 2 != 0) return OR_ARGUMENT_EXCEPTION;
        int64_t c = n / 2;
        if (dst_len < c) return OR_ARGUMENT_EXCEPTION;
        for (int64_t i = 0; i < c; i++) dst[i] = or_half_to_float(rd16(src + 2 * i));
        return OR_OK;
    }
    case 30: { /* DequantizeBF16 :120-137 */
        if (n % 2 != 0) return OR_ARGUMENT_EXCEPTION;
        int64_t c = n / 2;
        if (dst_len < c) return OR_ARGUMENT_EXCEPTION;
        for (int64_t i = 0; i < c; i++) dst[i] = or_bf16_to_float(rd16(src + 2 * i));
        return OR_OK;
    }
    case 2: { /* DequantizeQ4_0 :155-185 */
        if (n % 18 != 0) return OR_ARGUMENT_EXCEPTION;
        int64_t nb = n / 18;
        if (dst_len < nb * 32) return OR_ARGUMENT_EXCEPTION;
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* blk = src + b * 18;
            float d = or_half_to_float(rd16(blk));
            float* o = dst + b * 32;
            for (int j = 0; j < 16; j++) {
                uint8_t qs = blk[2 + j];
                o[j] = (float)((qs & 0x0F) - 8) * d;
                o[j + 16] = (float)((qs >> 4) - 8) * d;
            }
        }
        return OR_OK;
    }
    case 8: { /* DequantizeQ8_0 :203-231 */
        if (n % 34 != 0) return OR_ARGUMENT_EXCEPTION;
        int64_t nb = n / 34;
        if (dst_len < nb * 32) return OR_ARGUMENT_EXCEPTION;
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* blk = src + b * 34;
            float d = or_half_to_float(rd16(blk));
            float* o = dst + b * 32;
            for (int j = 0; j < 32; j++) o[j] = (float)(int8_t)blk[2 + j] * d;
        }
        return OR_OK;
    }
    case 12: { /* DequantizeQ4_K :251-294 */
        if (n % 144 != 0) return OR_ARGUMENT_EXCEPTION;
        int64_t nb = n / 144;
        if (dst_len < nb * 256) return OR_ARGUMENT_EXCEPTION;
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* blk = src + b * 144;
            float d = or_half_to_float(rd16(blk));
            float dmin = or_half_to_float(rd16(blk + 2));
            const uint8_t* scales = blk + 4;
            const uint8_t* qs = blk + 16;
            float* o = dst + b * 256;
            for (int g = 0; g < 8; g++) {
                int sc, mn;
                decode_kscale_min(scales, g, &sc, &mn);
                float dg = d * (float)sc;
                float mg = dmin * (float)mn;
                for (int i = 0; i < 32; i++) {
                    uint8_t packed = qs[g * 16 + (i >> 1)];
                    int q = (i & 1) == 0 ? (packed & 0x0F) : (packed >> 4);
                    o[g * 32 + i] = dg * (float)q - mg;
                }
            }
        }
        return OR_OK;
    }
    case 13: { /* DequantizeQ5_K :316-368 */
        if (n % 176 != 0) return OR_ARGUMENT_EXCEPTION;
        int64_t nb = n / 176;
        if (dst_len < nb * 256) return OR_ARGUMENT_EXCEPTION;
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* blk = src + b * 176;
            float d = or_half_to_float(rd16(blk));
            float dmin = or_half_to_float(rd16(blk + 2));
            const uint8_t* scales = blk + 4;
            const uint8_t* qh = blk + 16;
            const uint8_t* qs = blk + 48;
            float* o = dst + b * 256;
            for (int g = 0; g < 8; g++) {
                int sc, mn;
                decode_kscale_min(scales, g, &sc, &mn);
                float dg = d * (float)sc;
                float mg = dmin * (float)mn;
                for (int i = 0; i < 32; i++) {
                    int e = g * 32 + i;
                    uint8_t pl = qs[e >> 1];
                    int lo = (e & 1) == 0 ? (pl & 0x0F) : (pl >> 4);
                    int hi = (qh[e >> 3] >> (e & 7)) & 1;
                    int q = (hi << 4) | lo;
                    o[e] = dg * (float)q - mg;
                }
            }
        }
        return OR_OK;
    }
    case 14: { /* DequantizeQ6_K :378-417 */
        if (n % 210 != 0) return OR_ARGUMENT_EXCEPTION;
        int64_t nb = n / 210;
        if (dst_len < nb * 256) return OR_ARGUMENT_EXCEPTION;
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* blk = src + b * 210;
            const uint8_t* ql = blk;
            const uint8_t* qh = blk + 128;
            const uint8_t* sc = blk + 192;
            float d = or_half_to_float(rd16(blk + 208));
            float* o = dst + b * 256;
            for (int i = 0; i < 256; i++) {
                uint8_t qlb = ql[i >> 1];
                int lo = (i & 1) == 0 ? (qlb & 0x0F) : (qlb >> 4);
                int hi = (qh[i >> 2] >> ((i & 3) * 2)) & 3;
                int q = ((hi << 4) | lo) - 32;
                int s = (int8_t)sc[i >> 4];
                /* `d * scale * q` evaluates left to right: (d*scale)*q */
                o[i] = (d * (float)s) * (float)q;
            }
        }
        return OR_OK;
    }
    case 15: { /* DequantizeQ8_K :427-456 */
        if (n % 292 != 0) return OR_ARGUMENT_EXCEPTION;
        int64_t nb = n / 292;
        if (dst_len < nb * 256) return OR_ARGUMENT_EXCEPTION;
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* blk = src + b * 292;
            float d = bits_to_f32(rd32(blk));
            float* o = dst + b * 256;
            for (int i = 0; i < 256; i++) o[i] = (float)(int8_t)blk[4 + i] * d;
        }
        return OR_OK;
    }
    default:
        return OR_NOT_SUPPORTED;
    }
}

/* ════════════════════════════════════════════════════════════════════════
 * Tensors/TensorOperations.cs
 * ════════════════════════════════════════════════════════════════════════ */

/* TensorPrimitives.Dot (TensorOperations.cs:170-171): 8 partial sums (the
 * Vector256 accumulator shape), products rounded before the add. */
float or_dot(const float* a, const float* b, int n)
{
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int j = 0; j < 8; j++) {
            float p = a[i + j] * b[i + j];
            acc[j] = acc[j] + p;
        }
    float s = ((acc[0] + acc[4]) + (acc[1] + acc[5])) + ((acc[2] + acc[6]) + (acc[3] + acc[7]));
    for (; i < n; i++) {
        float p = a[i] * b[i];
        s = s + p;
    }
    return s;
}

/* TensorOperations.RmsNorm (TensorOperations.cs:42-54). */
void or_rmsnorm(const float* x, const float* w, float* dst, int n, float eps)
{
    float sum_sq = or_dot(x, x, n);
    float rms = 1.0f / sqrtf(sum_sq / (float)n + eps);
    for (int i = 0; i < n; i++) dst[i] = x[i] * rms;
    for (int i = 0; i < n; i++) dst[i] = dst[i] * w[i];
}

/* TensorOperations.GemmaRmsNorm (TensorOperations.cs:90-107): eps fixed 1e-6,
 * dst = (x*rms) * (1 + w).  x and dst may alias. */
void or_gemma_rmsnorm(const float* x, const float* w, float* dst, int n)
{
    float sum_sq = or_dot(x, x, n);
    float rms = 1.0f / sqrtf(sum_sq / (float)n + 1e-6f);
    for (int i = 0; i < n; i++) {
        float t = x[i] * rms;
        float one_w = w[i] + 1.0f;
        dst[i] = t * one_w;
    }
}

/* TensorOperations.Softmax (TensorOperations.cs:23-39). */
void or_softmax(float* x, int n)
{
    if (n == 0) return;
    float mx = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > mx || isnan(x[i])) mx = x[i];
    for (int i = 0; i < n; i++) x[i] = x[i] + (-mx);
    for (int i = 0; i < n; i++) x[i] = expf(x[i]);
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum = sum + x[i];
    if (sum != 0.0f)
        for (int i = 0; i < n; i++) x[i] = x[i] / sum;
}

/* TensorOperations.Silu (TensorOperations.cs:57-87): x * sigmoid(x),
 * sigmoid = 1 / (1 + exp(-x)). */
void or_silu(float* x, int n)
{
    for (int i = 0; i < n; i++) {
        float sig = 1.0f / (1.0f + expf(-x[i]));
        x[i] = x[i] * sig;
    }
}

/* TensorOperations.Gelu (TensorOperations.cs:110-117), tanh approximation. */
void or_gelu(float* x, int n)
{
    for (int i = 0; i < n; i++) {
        float v = x[i];
        float cube = ((0.044715f * v) * v) * v;
        float inner = 0.7978845608f * (v + cube);
        x[i] = (0.5f * v) * (1.0f + tanhf(inner));
    }
}

/* TensorOperations.SoftCap (TensorOperations.cs:120-126). */
void or_softcap(float* x, int n, float cap)
{
    float inv = 1.0f / cap;
    for (int i = 0; i < n; i++) x[i] = x[i] * inv;
    for (int i = 0; i < n; i++) x[i] = tanhf(x[i]);
    for (int i = 0; i < n; i++) x[i] = x[i] * cap;
}

/* TensorOperations.ArgMax → TensorPrimitives.IndexOfMax (TensorOperations.cs:
 * 187-195): the first index of the maximum; a NaN wins at its first position;
 * +0 ranks above -0. */
int or_argmax(const float* x, int n)
{
    if (n <= 0) return OR_ARGUMENT_EXCEPTION;
    int best = 0;
    float bv = x[0];
    if (isnan(bv)) return 0;
    for (int i = 1; i < n; i++) {
        float v = x[i];
        if (isnan(v)) return i;
        if (v > bv || (v == bv && v == 0.0f && signbit(bv) && !signbit(v))) {
            bv = v;
            best = i;
        }
    }
    return best;
}

static int cmp_desc(const void* a, const void* b)
{
    float x = *(const float*)a, y = *(const float*)b;
    return (x < y) - (x > y);
}

/* TopKSampler.ApplyTopK (TopKSampler.cs:42-71 of Sampling): values strictly
 * below the k-th largest become -inf; ties at the threshold are kept. */
void or_apply_topk(float* logits, int n, int k)
{
    if (k >= n) return;
    float* tmp = (float*)malloc(sizeof(float) * (size_t)n);
    memcpy(tmp, logits, sizeof(float) * (size_t)n);
    qsort(tmp, (size_t)n, sizeof(float), cmp_desc);
    float thr = tmp[k - 1];
    free(tmp);
    for (int i = 0; i < n; i++)
        if (logits[i] < thr) logits[i] = -INFINITY;
}

/* ── sampling ───────────────────────────────────────────────────────────── */

/* XoshiroRandom (Core/XoshiroRandom.cs:9-25): the 256-bit state from four
 * SplitMix64 outputs of the seed. */
static uint64_t splitmix64(uint64_t* x)
{
    *x += 0x9e3779b97f4a7c15ULL;
    uint64_t z = *x;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

void or_xoshiro_seed(uint64_t seed, uint64_t* st)
{
    for (int i = 0; i < 4; i++) st[i] = splitmix64(&seed);
}

static inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

/* XoshiroRandom.NextUInt64 (:28-39), xoshiro256**. */
uint64_t or_xoshiro_next(uint64_t* st)
{
    const uint64_t result = rotl64(st[1] * 5, 7) * 9;
    const uint64_t t = st[1] << 17;
    st[2] ^= st[0];
    st[3] ^= st[1];
    st[1] ^= st[2];
    st[0] ^= st[3];
    st[2] ^= t;
    st[3] = rotl64(st[3], 45);
    return result;
}

/* XoshiroRandom.NextFloat (:44): the top 53 bits as a double in [0, 1), then
 * rounded to float (which can round up to 1.0f). */
float or_xoshiro_next_float(uint64_t* st)
{
    return (float)((double)(or_xoshiro_next(st) >> 11) * (1.0 / 9007199254740992.0));
}

/* LlamaLanguageModel.ApplyRepetitionPenalty (LlamaLanguageModel.cs:357-373):
 * every occurrence in the generated list, in order: positive logits divided,
 * the others multiplied. */
void or_apply_repetition_penalty(float* logits, int n, const int* generated, int n_generated, float penalty)
{
    for (int i = 0; i < n_generated; i++) {
        const int id = generated[i];
        if ((unsigned)id < (unsigned)n) {
            if (logits[id] > 0.0f) logits[id] = logits[id] / penalty;
            else logits[id] = logits[id] * penalty;
        }
    }
}

static const float* g_topp_probs;
static int cmp_prob_desc(const void* a, const void* b)
{
    const int ia = *(const int*)a, ib = *(const int*)b;
    const float pa = g_topp_probs[ia], pb = g_topp_probs[ib];
    if (pa != pb) return pa < pb ? 1 : -1;
    return (ia > ib) - (ia < ib);
}

/* TopPSampler.ApplyTopP (TopPSampler.cs:60-110): walk the tokens by
 * descending probability, keep them until the running sum reaches p, zero the
 * rest, renormalize.  Ties are ordered by index (Array.Sort's introsort leaves
 * their order unspecified). */
void or_apply_topp(float* probs, int n, float p)
{
    if (p >= 1.0f) return;
    int* idx = (int*)malloc(sizeof(int) * (size_t)n);
    float* copy = (float*)malloc(sizeof(float) * (size_t)n);
    for (int i = 0; i < n; i++) idx[i] = i;
    memcpy(copy, probs, sizeof(float) * (size_t)n);
    g_topp_probs = copy;
    qsort(idx, (size_t)n, sizeof(int), cmp_prob_desc);
    float cum = 0.0f;
    int reached = 0;
    for (int r = 0; r < n; r++) {
        if (reached) {
            probs[idx[r]] = 0.0f;
        } else {
            cum = cum + probs[idx[r]];
            if (cum >= p) reached = 1;
        }
    }
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum = sum + probs[i];
    if (sum > 0.0f)
        for (int i = 0; i < n; i++) probs[i] = probs[i] / sum;
    free(idx);
    free(copy);
}

/* TemperatureSampler.SampleFromProbabilities (TemperatureSampler.cs:53-70). */
int or_sample_from_probs(const float* probs, int n, float u)
{
    float cum = 0.0f;
    for (int i = 0; i < n; i++) {
        cum = cum + probs[i];
        if (u < cum) return i;
    }
    for (int i = n - 1; i >= 0; i--)
        if (probs[i] > 0.0f) return i;
    return n - 1;
}

/* SamplerPipeline.Sample (SamplerPipeline.cs:58-89). */
int or_sampler_pipeline(float* logits, int n, float temperature, int top_k, float top_p, float u)
{
    if (temperature == 0.0f) return or_argmax(logits, n);
    if (temperature != 1.0f) {
        const float inv = 1.0f / temperature;
        for (int i = 0; i < n; i++) logits[i] = logits[i] * inv;
    }
    if (top_k > 0) or_apply_topk(logits, n, top_k);
    or_softmax(logits, n);
    if (top_p < 1.0f) or_apply_topp(logits, n, top_p);
    return or_sample_from_probs(logits, n, u);
}

/* TensorOperations.ApplyRope(Span<float>, float, ReadOnlySpan<float>)
 * (TensorOperations.cs:250-260): adjacent pairs rotated by pos*invFreq[i]. */
void or_rope(float* x, float position, const float* inv, int half)
{
    for (int i = 0; i < half; i++) {
        float theta = position * inv[i];
        float c = cosf(theta), s = sinf(theta);
        float x0 = x[2 * i], x1 = x[2 * i + 1];
        float a = x0 * c, b = x1 * s;
        float e = x0 * s, f = x1 * c;
        x[2 * i] = a - b;
        x[2 * i + 1] = e + f;
    }
}

/* ════════════════════════════════════════════════════════════════════════
 * ModelFormats.Gguf/GgufReader.cs + GgufFile.cs
 * ════════════════════════════════════════════════════════════════════════ */

enum { VT_U8 = 0, VT_I8, VT_U16, VT_I16, VT_U32, VT_I32, VT_F32, VT_BOOL, VT_STR, VT_ARR, VT_U64, VT_I64, VT_F64 };

typedef struct {
    char* key;
    int type;
    int arr_type;
    uint64_t arr_count;
    uint64_t u;   /* unsigned / bool payload */
    int64_t i;    /* signed payload */
    float f32;
    double f64;
    char* str;
} or_kv;

typedef struct {
    char* name;
    int ndims;
    uint64_t dims[8];
    int type;
    uint64_t offset;
} or_tinfo;

struct or_gguf {
    const uint8_t* data;
    int64_t len;
    uint32_t version;
    int64_t n_kv, n_tensors;
    or_kv* kv;
    or_tinfo* ti;
    int64_t data_start;
};

typedef struct {
    const uint8_t* p;
    int64_t len, pos;
    int bad;
} rdr;

static int need(rdr* r, int64_t n)
{
    if (r->bad || n < 0 || r->pos + n > r->len) {
        r->bad = 1;
        return 0;
    }
    return 1;
}
static uint8_t r8(rdr* r) { return need(r, 1) ? r->p[r->pos++] : 0; }
static uint16_t r16(rdr* r) { if (!need(r, 2)) return 0; uint16_t v = rd16(r->p + r->pos); r->pos += 2; return v; }
static uint32_t r32(rdr* r) { if (!need(r, 4)) return 0; uint32_t v = rd32(r->p + r->pos); r->pos += 4; return v; }
static uint64_t r64(rdr* r) { if (!need(r, 8)) return 0; uint64_t v = rd64(r->p + r->pos); r->pos += 8; return v; }
static char* rstr(rdr* r)
{
    uint64_t n = r64(r);
    if (r->bad || n > (uint64_t)(r->len - r->pos)) { r->bad = 1; return NULL; }
    char* s = (char*)malloc((size_t)n + 1);
    memcpy(s, r->p + r->pos, (size_t)n);
    s[n] = 0;
    r->pos += (int64_t)n;
    return s;
}

/* ReadScalarValue (GgufReader.cs:227-243); fills kv, returns 0 on unknown type. */
static int read_scalar(rdr* r, int vt, or_kv* kv)
{
    kv->type = vt;
    switch (vt) {
    case VT_U8: kv->u = r8(r); break;
    case VT_I8: kv->i = (int8_t)r8(r); break;
    case VT_U16: kv->u = r16(r); break;
    case VT_I16: kv->i = (int16_t)r16(r); break;
    case VT_U32: kv->u = r32(r); break;
    case VT_I32: kv->i = (int32_t)r32(r); break;
    case VT_F32: kv->f32 = bits_to_f32(r32(r)); break;
    case VT_BOOL: kv->u = r8(r) != 0; break;
    case VT_STR: kv->str = rstr(r); break;
    case VT_U64: kv->u = r64(r); break;
    case VT_I64: kv->i = (int64_t)r64(r); break;
    case VT_F64: { uint64_t b = r64(r); memcpy(&kv->f64, &b, 8); break; }
    default: return 0;
    }
    return 1;
}

void or_gguf_free(or_gguf* g)
{
    if (!g) return;
    for (int64_t i = 0; i < g->n_kv; i++) { free(g->kv[i].key); free(g->kv[i].str); }
    for (int64_t i = 0; i < g->n_tensors; i++) free(g->ti[i].name);
    free(g->kv);
    free(g->ti);
    free(g);
}

/* GgufReader.Parse (GgufReader.cs:55-111). */
or_gguf* or_gguf_parse(const uint8_t* data, int64_t len, char* err, int errlen)
{
    rdr r = {data, len, 0, 0};
    if (!need(&r, 4) || memcmp(data, "GGUF", 4) != 0) {
        set_err(err, errlen, "Not a GGUF file: invalid magic bytes.");
        return NULL;
    }
    r.pos = 4;
    uint32_t version = r32(&r);
    if (r.bad || (version != 2 && version != 3)) {
        set_err(err, errlen, "Unsupported GGUF version %u. Expected 2 or 3.", version);
        return NULL;
    }
    uint64_t n_t = r64(&r), n_kv = r64(&r);
    if (r.bad || n_kv > (uint64_t)len || n_t > (uint64_t)len) {
        set_err(err, errlen, "Truncated GGUF header.");
        return NULL;
    }
    or_gguf* g = (or_gguf*)calloc(1, sizeof(or_gguf));
    g->data = data;
    g->len = len;
    g->version = version;
    g->kv = (or_kv*)calloc(n_kv ? n_kv : 1, sizeof(or_kv));
    g->ti = (or_tinfo*)calloc(n_t ? n_t : 1, sizeof(or_tinfo));
    for (uint64_t i = 0; i < n_kv && !r.bad; i++) {
        or_kv* kv = &g->kv[i];
        g->n_kv = (int64_t)i + 1;
        kv->key = rstr(&r);
        int vt = (int)r32(&r);
        if (vt == VT_ARR) { /* ReadMetadataValue Array branch :208-220 */
            int et = (int)r32(&r);
            uint64_t cnt = version >= 3 ? r64(&r) : r32(&r);
            kv->type = VT_ARR;
            kv->arr_type = et;
            kv->arr_count = cnt;
            for (uint64_t j = 0; j < cnt && !r.bad; j++) {
                or_kv tmp;
                memset(&tmp, 0, sizeof tmp);
                if (!read_scalar(&r, et, &tmp)) {
                    set_err(err, errlen, "Unsupported array element type: %d", et);
                    or_gguf_free(g);
                    return NULL;
                }
                free(tmp.str);
            }
        } else if (!read_scalar(&r, vt, kv)) {
            set_err(err, errlen, "Unknown GGUF metadata value type: %d", vt);
            or_gguf_free(g);
            return NULL;
        }
    }
    for (uint64_t i = 0; i < n_t && !r.bad; i++) { /* ReadTensorInfo :245-265 */
        or_tinfo* t = &g->ti[i];
        g->n_tensors = (int64_t)i + 1;
        t->name = rstr(&r);
        uint32_t nd = r32(&r);
        if (nd > 8) { r.bad = 1; break; }
        t->ndims = (int)nd;
        for (uint32_t d = 0; d < nd; d++) t->dims[d] = r64(&r);
        t->type = (int)r32(&r);
        t->offset = r64(&r);
    }
    if (r.bad) {
        set_err(err, errlen, "Truncated GGUF header.");
        or_gguf_free(g);
        return NULL;
    }
    int64_t alignment = 32; /* DefaultAlignment :14 */
    for (int64_t i = g->n_kv - 1; i >= 0; i--) {
        if (g->kv[i].key && strcmp(g->kv[i].key, "general.alignment") == 0) {
            if (g->kv[i].type == VT_U32 || g->kv[i].type == VT_U64) alignment = (int32_t)(uint32_t)g->kv[i].u;
            break;
        }
    }
    if (alignment == 0) {
        set_err(err, errlen, "Attempted to divide by zero (general.alignment = 0).");
        or_gguf_free(g);
        return NULL;
    }
    g->data_start = ((r.pos + alignment - 1) / alignment) * alignment;
    return g;
}

uint32_t or_gguf_version(const or_gguf* g) { return g->version; }
int64_t or_gguf_tensor_count(const or_gguf* g) { return g->n_tensors; }
int64_t or_gguf_kv_count(const or_gguf* g) { return g->n_kv; }
int64_t or_gguf_data_start(const or_gguf* g) { return g->data_start; }

int64_t or_gguf_find_tensor(const or_gguf* g, const char* name)
{
    /* GgufFile._tensorIndex: ToDictionary (duplicate names throw in C#; the
     * generator never writes duplicates). */
    for (int64_t i = 0; i < g->n_tensors; i++)
        if (strcmp(g->ti[i].name, name) == 0) return i;
    return -1;
}

/* GgufFile.ComputeByteSize (GgufFile.cs:100-123). */
static int64_t compute_byte_size(const or_tinfo* t)
{
    int64_t e = 1;
    for (int d = 0; d < t->ndims; d++) e *= (int64_t)t->dims[d];
    switch (t->type) {
    case 0: return e * 4;
    case 1: case 30: return e * 2;
    case 2: return e / 32 * 18;
    case 3: return e / 32 * 20;
    case 6: return e / 32 * 22;
    case 7: return e / 32 * 24;
    case 8: return e / 32 * 34;
    case 9: return e / 32 * 36;
    case 12: return e / 256 * 144;
    case 13: return e / 256 * 176;
    case 14: return e / 256 * 210;
    case 15: return e / 256 * 292;
    default: return -1;
    }
}

int or_gguf_tensor_info(const or_gguf* g, int64_t idx, int* type, int* ndims, uint64_t* dims4,
                        uint64_t* offset, int64_t* nbytes)
{
    if (idx < 0 || idx >= g->n_tensors) return OR_ARGUMENT_OUT_OF_RANGE;
    const or_tinfo* t = &g->ti[idx];
    *type = t->type;
    *ndims = t->ndims;
    for (int d = 0; d < 4; d++) dims4[d] = d < t->ndims ? t->dims[d] : 1;
    *offset = t->offset;
    *nbytes = compute_byte_size(t);
    return OR_OK;
}

/* GgufModelLoader metadata helpers (GgufModelLoader.cs:433-478). */
static const or_kv* kv_find(const or_gguf* g, const char* key)
{
    for (int64_t i = g->n_kv - 1; i >= 0; i--) /* later duplicates overwrite */
        if (g->kv[i].key && strcmp(g->kv[i].key, key) == 0) return &g->kv[i];
    return NULL;
}
static const char* get_string(const or_gguf* g, const char* key, const char* def)
{
    const or_kv* v = kv_find(g, key);
    return (v && v->type == VT_STR && v->str) ? v->str : def;
}
static uint64_t get_uint(const or_gguf* g, const char* key, uint64_t def, int array_length)
{
    const or_kv* v = kv_find(g, key);
    if (!v) return def;
    if (array_length && v->type == VT_ARR) return v->arr_count;
    switch (v->type) {
    case VT_U8: case VT_U16: case VT_U32: case VT_U64: return v->u;
    case VT_I32: case VT_I64: return (uint64_t)v->i;
    default: return def;
    }
}
static float get_float(const or_gguf* g, const char* key, float def)
{
    const or_kv* v = kv_find(g, key);
    return (v && v->type == VT_F32) ? v->f32 : def;
}

/* ════════════════════════════════════════════════════════════════════════
 * Architectures (Llama/Mistral/Gemma2/Qwen2 forward passes) + KvCache
 * ════════════════════════════════════════════════════════════════════════ */

enum { ARCH_LLAMA = 0, ARCH_MISTRAL = 1, ARCH_GEMMA2 = 2, ARCH_QWEN2 = 3 };

/* A weight matrix [rows, cols]: either dequantized once into F32 (`f`, the
 * reference's LoadTensor) or kept as the raw GGUF blocks of the image (`raw`)
 * and dequantized one row at a time where it is used.  A row of whole blocks
 * decodes to the same floats either way (every block is independent), so the
 * lazy form changes no value; it only keeps host memory at the size of the
 * quantized file (Llama-3-8B: 4.9 GB instead of ~32 GB of F32). */
typedef struct {
    float* f;
    const uint8_t* raw;
    int type;
    int64_t row_bytes;
} or_mat;

typedef struct {
    float *attn_norm, *ffn_norm;
    or_mat wq, wk, wv, wo, gate, up, down;
    float *post_attn_norm, *post_ffn_norm; /* gemma2 */
    float *bq, *bk, *bv;                   /* qwen2 */
} or_layer;

struct or_model {
    int arch;
    int n_layers, n_layers_loaded, hidden, ffn, n_heads, n_kv, head_dim, vocab, max_ctx, bos, eos;
    int window;           /* INT_MAX = none */
    float rope_base, rope_factor;
    int rope_scaled;      /* RopeScalingType is linear|yarn and factor > 0 */
    float attn_softcap, final_softcap, attn_scale;
    or_mat tok_embd;
    float* out_norm;
    or_mat output;        /* may alias tok_embd (tied) */
    or_layer* layers;
    float* inv_freq;      /* [head_dim/2] */
};

void or_model_free(or_model* m)
{
    if (!m) return;
    for (int l = 0; l < m->n_layers_loaded; l++) {
        or_layer* L = &m->layers[l];
        free(L->attn_norm); free(L->wq.f); free(L->wk.f); free(L->wv.f); free(L->wo.f);
        free(L->ffn_norm); free(L->gate.f); free(L->up.f); free(L->down.f);
        free(L->post_attn_norm); free(L->post_ffn_norm);
        free(L->bq); free(L->bk); free(L->bv);
    }
    free(m->layers);
    if (m->output.f != m->tok_embd.f) free(m->output.f);
    free(m->tok_embd.f);
    free(m->out_norm);
    free(m->inv_freq);
    free(m);
}

/* GgufModelLoader.LoadTensor / LoadTensorOptional (GgufModelLoader.cs:409-432). */
static float* load_tensor(const or_gguf* g, const char* name, int64_t expected, int optional, char* err, int errlen,
                          int* fail)
{
    int64_t idx = or_gguf_find_tensor(g, name);
    if (idx < 0) {
        if (!optional) {
            set_err(err, errlen, "Required tensor '%s' not found in GGUF file.", name);
            *fail = 1;
        }
        return NULL;
    }
    const or_tinfo* t = &g->ti[idx];
    int64_t nbytes = compute_byte_size(t);
    if (nbytes < 0) {
        set_err(err, errlen, "Cannot compute byte size for tensor type %d.", t->type);
        *fail = 1;
        return NULL;
    }
    int64_t abs_off = g->data_start + (int64_t)t->offset;
    if (abs_off < 0 || abs_off + nbytes > g->len) {
        set_err(err, errlen, "Tensor '%s' data lies outside the file.", name);
        *fail = 1;
        return NULL;
    }
    float* dst = (float*)calloc((size_t)(expected > 0 ? expected : 1), sizeof(float));
    int rc = or_dequantize(t->type, g->data + abs_off, nbytes, dst, expected);
    if (rc != OR_OK) {
        set_err(err, errlen, rc == OR_NOT_SUPPORTED ? "Tensor type %d is not supported for dequantization."
                                                    : "Destination too small for tensor type %d.", t->type);
        free(dst);
        *fail = 1;
        return NULL;
    }
    return dst;
}

/* Elements and bytes of one block of a dequantizable type (the block
 * constants of Dequantizer.cs:19-43); 0 for an unknown type. */
static int block_geom(int type, int* elems, int* bytes)
{
    switch (type) {
    case 0: *elems = 1; *bytes = 4; return 1;    /* F32 */
    case 1: *elems = 1; *bytes = 2; return 1;    /* F16 */
    case 30: *elems = 1; *bytes = 2; return 1;   /* BF16 */
    case 2: *elems = 32; *bytes = 18; return 1;  /* Q4_0 */
    case 8: *elems = 32; *bytes = 34; return 1;  /* Q8_0 */
    case 12: *elems = 256; *bytes = 144; return 1; /* Q4_K */
    case 13: *elems = 256; *bytes = 176; return 1; /* Q5_K */
    case 14: *elems = 256; *bytes = 210; return 1; /* Q6_K */
    case 15: *elems = 256; *bytes = 292; return 1; /* Q8_K */
    default: return 0;
    }
}

/* A [rows, cols] matrix: lazy (raw blocks of the image, decoded per row) when
 * asked and every row is a whole number of blocks, else load_tensor's F32. */
static or_mat load_matrix(const or_gguf* g, const char* name, int64_t rows, int64_t cols, int optional, int lazy,
                          char* err, int errlen, int* fail)
{
    or_mat mt = {NULL, NULL, 0, 0};
    int64_t idx = or_gguf_find_tensor(g, name);
    int be = 0, bb = 0;
    if (lazy && idx >= 0 && block_geom(g->ti[idx].type, &be, &bb) && cols % be == 0) {
        const or_tinfo* t = &g->ti[idx];
        const int64_t nbytes = compute_byte_size(t);
        const int64_t row_bytes = cols / be * bb;
        const int64_t abs_off = g->data_start + (int64_t)t->offset;
        if (nbytes == rows * row_bytes && abs_off >= 0 && abs_off + nbytes <= g->len) {
            mt.raw = g->data + abs_off;
            mt.type = t->type;
            mt.row_bytes = row_bytes;
            return mt;
        }
    }
    mt.f = load_tensor(g, name, rows * cols, optional, err, errlen, fail);
    return mt;
}

/* Row r of a matrix with `cols` columns into dst (F32). */
static void mat_row(const or_mat* w, int64_t r, int cols, float* dst)
{
    if (w->f) memcpy(dst, w->f + (size_t)r * cols, sizeof(float) * (size_t)cols);
    else or_dequantize(w->type, w->raw + r * w->row_bytes, w->row_bytes, dst, cols);
}

/* GgufModelLoader.Build/BuildConfig/BuildMistral/BuildGemma2/BuildQwen2 +
 * LoadWeights/LoadGemma2Weights/LoadQwen2Weights (GgufModelLoader.cs:89-372,
 * 518-590). */
or_model* or_model_load_ex(const uint8_t* data, int64_t len, int max_layers, int lazy, char* err, int errlen)
{
    char perr[256] = {0};
    or_gguf* g = or_gguf_parse(data, len, perr, sizeof perr);
    if (!g) {
        set_err(err, errlen, "%s", perr);
        return NULL;
    }
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    const char* arch = get_string(g, "general.architecture", "llama");
    char key[256];
#define K(suffix) (snprintf(key, sizeof key, "%s." suffix, pfx), key)
    const char* pfx = arch;
    if (!strcmp(arch, "llama") || !strcmp(arch, "llama3") || !strcmp(arch, "llama4")) m->arch = ARCH_LLAMA;
    else if (!strcmp(arch, "mistral")) m->arch = ARCH_MISTRAL;
    else if (!strcmp(arch, "gemma") || !strcmp(arch, "gemma2")) m->arch = ARCH_GEMMA2;
    else if (!strcmp(arch, "qwen2")) m->arch = ARCH_QWEN2;
    else {
        set_err(err, errlen, "Architecture '%s' is not supported. Supported: llama, mistral, gemma2, qwen2.", arch);
        or_gguf_free(g);
        free(m);
        return NULL;
    }
    if (m->arch == ARCH_GEMMA2) pfx = kv_find(g, "gemma2.block_count") ? "gemma2" : "gemma";

    int head_dim_override = m->arch == ARCH_GEMMA2 ? (int)get_uint(g, K("attention.key_length"), 0, 0) : 0;
    m->n_layers = (int)get_uint(g, K("block_count"), 0, 0);
    m->hidden = (int)get_uint(g, K("embedding_length"), 0, 0);
    m->ffn = (int)get_uint(g, K("feed_forward_length"), 0, 0);
    m->n_heads = (int)get_uint(g, K("attention.head_count"), 0, 0);
    uint64_t hc = get_uint(g, K("attention.head_count"), 0, 0);
    m->n_kv = (int)get_uint(g, K("attention.head_count_kv"), hc, 0);
    m->max_ctx = (int)get_uint(g, K("context_length"), 4096, 0);
    uint64_t vdef = get_uint(g, "tokenizer.ggml.tokens", 32000, 1);
    m->vocab = (int)get_uint(g, K("vocab_size"), vdef, 0);
    m->rope_base = get_float(g, K("rope.freq_base"), 10000.0f);
    float fs = get_float(g, K("rope.freq_scale"), 1.0f);
    m->rope_factor = get_float(g, K("rope.scaling.factor"), fs);
    const char* rst = get_string(g, K("rope.scaling.type"), "none");
    m->rope_scaled = (!strcasecmp(rst, "linear") || !strcasecmp(rst, "yarn")) && m->rope_factor > 0.0f;
    m->bos = (int)get_uint(g, "tokenizer.ggml.bos_token_id", 1, 0);
    m->eos = (int)get_uint(g, "tokenizer.ggml.eos_token_id", 2, 0);
    m->window = INT_MAX;
    m->head_dim = m->n_heads > 0 ? m->hidden / m->n_heads : 0;
    m->attn_scale = m->head_dim > 0 ? 1.0f / sqrtf((float)m->head_dim) : 0.0f;
    if (m->arch == ARCH_MISTRAL)
        m->window = (int)get_uint(g, "mistral.attention.sliding_window", (uint64_t)INT_MAX, 0);
    if (m->arch == ARCH_GEMMA2) {
        m->head_dim = head_dim_override > 0 ? head_dim_override : (m->n_heads > 0 ? m->hidden / m->n_heads : 0);
        m->window = (int)get_uint(g, K("attention.sliding_window"), (uint64_t)INT_MAX, 0);
        m->attn_softcap = get_float(g, K("attn_logit_softcapping"), 0.0f);
        m->final_softcap = get_float(g, K("final_logit_softcapping"), 0.0f);
        m->attn_scale = get_float(g, K("attention.query_pre_attn_scalar"), 1.0f / sqrtf((float)m->head_dim));
    }
    /* Forward-pass constructor check (LlamaForwardPass.cs:48-52). */
    if (m->n_kv <= 0 || m->n_heads <= 0 || m->n_kv > m->n_heads || (m->n_heads % m->n_kv) != 0 ||
        m->head_dim <= 0 || (m->head_dim & 1)) {
        set_err(err, errlen, "Invalid attention head configuration: NumHeads=%d, NumKvHeads=%d.", m->n_heads, m->n_kv);
        or_gguf_free(g);
        free(m);
        return NULL;
    }

    int h = m->hidden, qd = m->n_heads * m->head_dim, kvd = m->n_kv * m->head_dim, f = m->ffn, V = m->vocab;
    int fail = 0;
    m->n_layers_loaded = (max_layers >= 0 && max_layers < m->n_layers) ? max_layers : m->n_layers;
    m->tok_embd = load_matrix(g, "token_embd.weight", V, h, 0, lazy, err, errlen, &fail);
    m->layers = (or_layer*)calloc((size_t)(m->n_layers_loaded > 0 ? m->n_layers_loaded : 1), sizeof(or_layer));
    for (int l = 0; l < m->n_layers_loaded && !fail; l++) {
        or_layer* L = &m->layers[l];
        char nm[128];
#define LT(field, suffix, cnt)                                                        \
    do {                                                                              \
        snprintf(nm, sizeof nm, "blk.%d." suffix, l);                                 \
        if (!fail) L->field = load_tensor(g, nm, (int64_t)(cnt), 0, err, errlen, &fail); \
    } while (0)
#define LM(field, suffix, r, c)                                                                   \
    do {                                                                                          \
        snprintf(nm, sizeof nm, "blk.%d." suffix, l);                                             \
        if (!fail) L->field = load_matrix(g, nm, (int64_t)(r), (int64_t)(c), 0, lazy, err, errlen, &fail); \
    } while (0)
        LT(attn_norm, "attn_norm.weight", h);
        if (m->arch == ARCH_GEMMA2) LT(post_attn_norm, "post_attn_norm.weight", h);
        LM(wq, "attn_q.weight", qd, h);
        LM(wk, "attn_k.weight", kvd, h);
        LM(wv, "attn_v.weight", kvd, h);
        LM(wo, "attn_output.weight", h, qd);
        if (m->arch == ARCH_QWEN2) {
            LT(bq, "attn_q.bias", qd);
            LT(bk, "attn_k.bias", kvd);
            LT(bv, "attn_v.bias", kvd);
        }
        LT(ffn_norm, "ffn_norm.weight", h);
        if (m->arch == ARCH_GEMMA2) LT(post_ffn_norm, "post_ffn_norm.weight", h);
        LM(gate, "ffn_gate.weight", f, h);
        LM(up, "ffn_up.weight", f, h);
        LM(down, "ffn_down.weight", h, f);
#undef LT
#undef LM
    }
    if (!fail) m->out_norm = load_tensor(g, "output_norm.weight", h, 0, err, errlen, &fail);
    if (!fail) {
        m->output = load_matrix(g, "output.weight", V, h, 1, lazy, err, errlen, &fail);
        if (!m->output.f && !m->output.raw && !fail) m->output = m->tok_embd;
    }
#undef K
    or_gguf_free(g);
    if (fail) {
        or_model_free(m);
        return NULL;
    }
    int half = m->head_dim / 2;
    m->inv_freq = (float*)malloc(sizeof(float) * (size_t)half);
    for (int i = 0; i < half; i++) { /* LlamaForwardPass.cs:64-70 */
        float ex = (2.0f * (float)i) / (float)m->head_dim;
        m->inv_freq[i] = 1.0f / powf(m->rope_base, ex);
    }
    return m;
}

or_model* or_model_load(const uint8_t* data, int64_t len, int max_layers, char* err, int errlen)
{
    return or_model_load_ex(data, len, max_layers, 0, err, errlen);
}

void or_model_config(const or_model* m, int* arch, int* iv, float* fv)
{
    *arch = m->arch;
    iv[0] = m->n_layers; iv[1] = m->hidden; iv[2] = m->ffn; iv[3] = m->n_heads; iv[4] = m->n_kv;
    iv[5] = m->head_dim; iv[6] = m->vocab; iv[7] = m->max_ctx; iv[8] = m->bos; iv[9] = m->eos;
    iv[10] = m->window; iv[11] = m->rope_scaled;
    fv[0] = m->rope_base; fv[1] = m->rope_factor; fv[2] = m->attn_softcap; fv[3] = m->final_softcap;
    fv[4] = m->attn_scale; fv[5] = 0; fv[6] = 0; fv[7] = 0;
}

/* Inference/KvCache.cs restated (Append :59-97, GetKeys :100-116, Evict :152-173). */
typedef struct {
    int layers, max_seq, kv_dim, cur, next_layer, evicted;
    float **keys, **values;
} or_kvcache;

static void kv_init(or_kvcache* c, int layers, int max_seq, int kv_dim)
{
    c->layers = layers; c->max_seq = max_seq; c->kv_dim = kv_dim;
    c->cur = 0; c->next_layer = 0; c->evicted = 0;
    c->keys = (float**)calloc((size_t)layers, sizeof(float*));
    c->values = (float**)calloc((size_t)layers, sizeof(float*));
    for (int l = 0; l < layers; l++) {
        c->keys[l] = (float*)calloc((size_t)max_seq * kv_dim, sizeof(float));
        c->values[l] = (float*)calloc((size_t)max_seq * kv_dim, sizeof(float));
    }
}
static void kv_free(or_kvcache* c)
{
    for (int l = 0; l < c->layers; l++) { free(c->keys[l]); free(c->values[l]); }
    free(c->keys);
    free(c->values);
}
static void kv_evict_oldest_half(or_kvcache* c)
{
    int retained = c->max_seq / 2;
    size_t src = (size_t)retained * c->kv_dim;
    size_t copy_len = (size_t)(c->max_seq - retained) * c->kv_dim;
    for (int l = 0; l < c->layers; l++) {
        memmove(c->keys[l], c->keys[l] + src, copy_len * sizeof(float));
        memset(c->keys[l] + copy_len, 0, src * sizeof(float));
        memmove(c->values[l], c->values[l] + src, copy_len * sizeof(float));
        memset(c->values[l] + copy_len, 0, src * sizeof(float));
    }
    c->cur = retained;
    c->evicted = 1;
}
static int kv_append(or_kvcache* c, int layer, const float* k, const float* v)
{
    if (layer < 0 || layer >= c->layers) return OR_ARGUMENT_OUT_OF_RANGE;
    if (layer != c->next_layer) return OR_INVALID_OPERATION;
    if (c->cur >= c->max_seq) kv_evict_oldest_half(c);
    size_t off = (size_t)c->cur * c->kv_dim;
    memcpy(c->keys[layer] + off, k, sizeof(float) * (size_t)c->kv_dim);
    memcpy(c->values[layer] + off, v, sizeof(float) * (size_t)c->kv_dim);
    c->next_layer++;
    if (c->next_layer == c->layers) { c->next_layer = 0; c->cur++; }
    return OR_OK;
}
static int kv_effective_length(const or_kvcache* c, int layer)
{
    int e = c->cur;
    if (c->next_layer > 0 && layer < c->next_layer) e++;
    return e;
}

struct or_session {
    or_model* m;
    or_kvcache kv;
    float *x, *xn, *q, *k, *v, *att, *ffn_buf, *ffn_up, *logits, *scores;
};

or_session* or_session_create(or_model* m)
{
    or_session* s = (or_session*)calloc(1, sizeof(or_session));
    s->m = m;
    int qd = m->n_heads * m->head_dim, kvd = m->n_kv * m->head_dim;
    /* LlamaLanguageModel.cs:129: new KvCache(layers, maxContextLength, kvDim). */
    kv_init(&s->kv, m->n_layers, m->max_ctx, kvd);
    s->x = (float*)calloc((size_t)m->hidden, 4);
    s->xn = (float*)calloc((size_t)m->hidden, 4);
    s->q = (float*)calloc((size_t)qd, 4);
    s->k = (float*)calloc((size_t)kvd, 4);
    s->v = (float*)calloc((size_t)kvd, 4);
    s->att = (float*)calloc((size_t)qd, 4);
    s->ffn_buf = (float*)calloc((size_t)m->ffn, 4);
    s->ffn_up = (float*)calloc((size_t)m->ffn, 4);
    s->logits = (float*)calloc((size_t)m->vocab, 4);
    s->scores = (float*)calloc((size_t)m->max_ctx + 1, 4);
    return s;
}

void or_session_free(or_session* s)
{
    if (!s) return;
    kv_free(&s->kv);
    free(s->x); free(s->xn); free(s->q); free(s->k); free(s->v); free(s->att);
    free(s->ffn_buf); free(s->ffn_up); free(s->logits); free(s->scores);
    free(s);
}

int or_session_length(const or_session* s) { return s->kv.cur; }

/* Timing samples only: marks the first n positions of the KV cache as filled
 * (their contents stay as they are), so a forward at position n attends over
 * n+1 keys without running n earlier forwards. */
int or_session_fake_length(or_session* s, int n)
{
    if (n < 0 || n >= s->kv.max_seq) return OR_ARGUMENT_OUT_OF_RANGE;
    s->kv.cur = n;
    s->kv.next_layer = 0;
    return OR_OK;
}

/* LinearProjection (LlamaForwardPass.cs:237-260): dst[o] = Dot(src, W[o,:]).
 * Rows are independent, so the OpenMP split does not change any value. */
static void linear(const float* src, const or_mat* w, float* dst, int out_dim, int in_dim)
{
    if (w->f) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
        for (int o = 0; o < out_dim; o++) dst[o] = or_dot(src, w->f + (size_t)o * in_dim, in_dim);
        return;
    }
#pragma omp parallel num_threads(g_threads) if (g_threads > 1)
    {
        float* row = (float*)malloc(sizeof(float) * (size_t)in_dim);
#pragma omp for schedule(static)
        for (int o = 0; o < out_dim; o++) {
            mat_row(w, o, in_dim, row);
            dst[o] = or_dot(src, row, in_dim);
        }
        free(row);
    }
}

static void rope_all_heads(const or_model* m, float* vec, int position, int n_heads)
{
    /* ApplyRopeAllHeads (LlamaForwardPass.cs:135-148). */
    float pos = m->rope_scaled ? (float)position / m->rope_factor : (float)position;
    for (int h = 0; h < n_heads; h++) or_rope(vec + (size_t)h * m->head_dim, pos, m->inv_freq, m->head_dim / 2);
}

/* ComputeAttention (LlamaForwardPass.cs:158-211; MistralForwardPass.cs:186-240;
 * Gemma2ForwardPass.cs:126-185; Qwen2ForwardPass.cs:124-175). */
static int attention(or_session* s, int layer, int seq_len, int window)
{
    or_model* m = s->m;
    int hd = m->head_dim, nh = m->n_heads, nkv = m->n_kv, grp = nh / nkv, kvd = nkv * hd;
    int eff = kv_effective_length(&s->kv, layer);
    int wstart = seq_len - window;
    if (window == INT_MAX || wstart < 0) wstart = 0;
    if (seq_len > eff) return OR_ARGUMENT_OUT_OF_RANGE; /* span slice past the cache */
    int att_len = seq_len - wstart;
    const float* K = s->kv.keys[layer];
    const float* V = s->kv.values[layer];
    memset(s->att, 0, sizeof(float) * (size_t)nh * hd);
    for (int qh = 0; qh < nh; qh++) {
        int kvh = qh / grp;
        const float* q = s->q + (size_t)qh * hd;
        for (int t = wstart; t < seq_len; t++)
            s->scores[t - wstart] = or_dot(q, K + (size_t)t * kvd + (size_t)kvh * hd, hd) * m->attn_scale;
        if (m->arch == ARCH_GEMMA2 && m->attn_softcap > 0.0f) or_softcap(s->scores, att_len, m->attn_softcap);
        or_softmax(s->scores, att_len);
        float* out = s->att + (size_t)qh * hd;
        for (int t = wstart; t < seq_len; t++) {
            const float* v = V + (size_t)t * kvd + (size_t)kvh * hd;
            float w = s->scores[t - wstart];
            for (int d = 0; d < hd; d++) {
                float p = v[d] * w;
                out[d] = out[d] + p;
            }
        }
    }
    return OR_OK;
}

static int forward_layers(or_session* s, int token, int position, int n_layers)
{
    or_model* m = s->m;
    int h = m->hidden, qd = m->n_heads * m->head_dim, kvd = m->n_kv * m->head_dim, f = m->ffn;
    if ((unsigned)token >= (unsigned)m->vocab) return OR_ARGUMENT_OUT_OF_RANGE; /* :89-93 */
    mat_row(&m->tok_embd, token, h, s->x);   /* :96 */
    int gemma = m->arch == ARCH_GEMMA2;
    for (int l = 0; l < n_layers; l++) {
        or_layer* L = &m->layers[l];
        if (gemma) or_gemma_rmsnorm(s->x, L->attn_norm, s->xn, h);
        else or_rmsnorm(s->x, L->attn_norm, s->xn, h, 1e-5f);
        linear(s->xn, &L->wq, s->q, qd, h);
        linear(s->xn, &L->wk, s->k, kvd, h);
        linear(s->xn, &L->wv, s->v, kvd, h);
        if (m->arch == ARCH_QWEN2) { /* Qwen2ForwardPass.cs:83-85 */
            for (int i = 0; i < qd; i++) s->q[i] = s->q[i] + L->bq[i];
            for (int i = 0; i < kvd; i++) s->k[i] = s->k[i] + L->bk[i];
            for (int i = 0; i < kvd; i++) s->v[i] = s->v[i] + L->bv[i];
        }
        rope_all_heads(m, s->q, position, m->n_heads);
        rope_all_heads(m, s->k, position, m->n_kv);
        int rc = kv_append(&s->kv, l, s->k, s->v);
        if (rc) return rc;
        int window = INT_MAX;
        if (m->arch == ARCH_MISTRAL) window = m->window;
        if (gemma) window = (l % 2 == 0) ? m->window : INT_MAX; /* Gemma2ForwardPass.cs:87 */
        rc = attention(s, l, position + 1, window);
        if (rc) return rc;
        linear(s->att, &L->wo, s->xn, h, qd);
        if (gemma) or_gemma_rmsnorm(s->xn, L->post_attn_norm, s->xn, h);
        for (int i = 0; i < h; i++) s->x[i] = s->x[i] + s->xn[i];
        if (gemma) or_gemma_rmsnorm(s->x, L->ffn_norm, s->xn, h);
        else or_rmsnorm(s->x, L->ffn_norm, s->xn, h, 1e-5f);
        /* ComputeSiluFfn (LlamaForwardPass.cs:217-232) / ComputeGeluFfn (Gemma2:187-199) */
        linear(s->xn, &L->gate, s->ffn_buf, f, h);
        if (gemma) or_gelu(s->ffn_buf, f);
        else or_silu(s->ffn_buf, f);
        linear(s->xn, &L->up, s->ffn_up, f, h);
        for (int i = 0; i < f; i++) s->ffn_buf[i] = s->ffn_buf[i] * s->ffn_up[i];
        linear(s->ffn_buf, &L->down, s->xn, h, f);
        if (gemma) or_gemma_rmsnorm(s->xn, L->post_ffn_norm, s->xn, h);
        for (int i = 0; i < h; i++) s->x[i] = s->x[i] + s->xn[i];
    }
    return OR_OK;
}

int or_forward_head(or_session* s, float* logits_out)
{
    or_model* m = s->m;
    int h = m->hidden;
    if (m->arch == ARCH_GEMMA2) or_gemma_rmsnorm(s->x, m->out_norm, s->xn, h);
    else or_rmsnorm(s->x, m->out_norm, s->xn, h, 1e-5f);
    linear(s->xn, &m->output, s->logits, m->vocab, h);
    if (m->arch == ARCH_GEMMA2 && m->final_softcap > 0.0f) or_softcap(s->logits, m->vocab, m->final_softcap);
    if (logits_out) memcpy(logits_out, s->logits, sizeof(float) * (size_t)m->vocab);
    return OR_OK;
}

int or_forward_layers(or_session* s, int token, int position, int n_layers)
{
    if (n_layers > s->m->n_layers_loaded) return OR_ARGUMENT_OUT_OF_RANGE;
    return forward_layers(s, token, position, n_layers);
}

/* IForwardPass.Forward (LlamaForwardPass.cs:82-130 and per-arch copies). */
int or_forward(or_session* s, int token, int position, float* logits_out)
{
    if (s->m->n_layers_loaded != s->m->n_layers) return OR_INVALID_OPERATION;
    int rc = forward_layers(s, token, position, s->m->n_layers);
    if (rc) return rc;
    return or_forward_head(s, logits_out);
}

/* LlamaLanguageModel.GenerateAsync with Temperature = 0 (LlamaLanguageModel.cs:
 * 126-293, SamplerPipeline.cs:79-82): prefill every prompt token but the last,
 * then forward the last prompt token as decode step 0; greedy ArgMax; stop at
 * EOS or after max_tokens.  Returns the number of generated tokens. */
int or_generate_greedy(or_model* m, const int* prompt, int n_prompt, int max_tokens, int* out_tokens,
                       float* out_logits)
{
    or_session* s = or_session_create(m);
    int pos = 0, rc = OR_OK;
    for (int i = 0; i < n_prompt - 1; i++) {
        rc = or_forward(s, prompt[i], pos++, NULL);
        if (rc) { or_session_free(s); return rc; }
    }
    int next = n_prompt > 0 ? prompt[n_prompt - 1] : m->bos;
    int n = 0;
    for (int step = 0; step < max_tokens; step++) {
        rc = or_forward(s, next, pos++, NULL);
        if (rc) { or_session_free(s); return rc; }
        if (out_logits) memcpy(out_logits + (size_t)step * m->vocab, s->logits, sizeof(float) * (size_t)m->vocab);
        next = or_argmax(s->logits, m->vocab);
        out_tokens[n++] = next;
        if (next == m->eos) break;
    }
    or_session_free(s);
    return n;
}
