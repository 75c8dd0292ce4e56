/*
 * ggufgen.c — seeded synthetic GGUF weights for the benchmark configurations.
 *
 * The reference ships no model files, so every model used by the tests and the
 * benchmark is random-init.  This file produces the tensor payloads:
 *
 *  - values: a counter-based normal stream.  Element i of stream s is the sum of
 *    twelve 16-bit uniforms drawn from splitmix64(seed, s, i) minus their mean
 *    (the classic "sum of 12 uniforms" approximation of N(0,1), exact in integer
 *    arithmetic, so every host produces identical floats), times sigma;
 *  - quantization: the inverse of the reference decoder
 *    (src/DotNetFoundryLLM.Quantization/Dequantizer.cs) — the sequential nibble
 *    and high-bit layouts that decoder reads (Dequantizer.cs:285-290, 353-363,
 *    404-414), its 6-bit scale/min packing (DecodeKScaleMin :506-521), fitted per
 *    group by min/max.  The quantizer only has to produce valid blocks: parity is
 *    defined on whatever bytes it writes, decoded by the reference rules.
 *
 * Host-only C; OpenMP splits the work by block, and every block depends only on
 * its own indices, so the output does not depend on the thread count.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_Q8_K = 15, T_BF16 = 30 };

static int g_threads = 0;
int gg_set_threads(int n) { g_threads = n; return 0; }
static int nthreads(void)
{
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

static inline uint64_t splitmix64(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static inline uint64_t stream_base(uint64_t seed, uint64_t stream) { return splitmix64(seed ^ splitmix64(stream)); }

/* Sum of twelve 16-bit uniforms, centred: an integer in [-393210, 393210]. */
static inline float normal_at(uint64_t base, int64_t i, float sigma)
{
    uint64_t h0 = splitmix64(base + 3ull * (uint64_t)i);
    uint64_t h1 = splitmix64(base + 3ull * (uint64_t)i + 1);
    uint64_t h2 = splitmix64(base + 3ull * (uint64_t)i + 2);
    int32_t s = 0;
    for (int k = 0; k < 4; k++) {
        s += (int32_t)((h0 >> (16 * k)) & 0xFFFF);
        s += (int32_t)((h1 >> (16 * k)) & 0xFFFF);
        s += (int32_t)((h2 >> (16 * k)) & 0xFFFF);
    }
    float z = (float)(s - 393210) * (1.0f / 65536.0f);
    return z * sigma;
}

void gg_normal_f32(uint64_t seed, uint64_t stream, int64_t start, int64_t n, float sigma, float* dst)
{
    uint64_t base = stream_base(seed, stream);
#pragma omp parallel for schedule(static) num_threads(nthreads())
    for (int64_t i = 0; i < n; i++) dst[i] = normal_at(base, start + i, sigma);
}

void gg_uniform_ids(uint64_t seed, uint64_t stream, int64_t n, int32_t vocab, int32_t* out)
{
    uint64_t base = stream_base(seed, stream);
    for (int64_t i = 0; i < n; i++) out[i] = (int32_t)(splitmix64(base + (uint64_t)i) % (uint64_t)vocab);
}

/* IEEE binary32 → binary16, round to nearest even. */
uint16_t gg_f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;
        uint32_t hm = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
    return (uint16_t)h;
}

float gg_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, out;
    if (exp == 0) {
        if (man == 0) out = sign;
        else {
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            out = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1F) out = sign | 0x7F800000u | (man << 13);
    else out = sign | ((exp + 112u) << 23) | (man << 13);
    float f;
    memcpy(&f, &out, 4);
    return f;
}

static uint16_t f32_to_bf16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

static inline void wr16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Encodes the 6-bit scale/min pairs so that DecodeKScaleMin returns them. */
static void pack_kscale_min(const int* sc, const int* mn, uint8_t* p)
{
    memset(p, 0, 12);
    for (int g = 0; g < 4; g++) {
        p[g] |= (uint8_t)(sc[g] & 63);
        p[g + 4] |= (uint8_t)(mn[g] & 63);
    }
    for (int g = 4; g < 8; g++) {
        p[g + 4] = (uint8_t)((sc[g] & 0xF) | ((mn[g] & 0xF) << 4));
        p[g - 4] |= (uint8_t)((sc[g] >> 4) << 6);
        p[g] |= (uint8_t)((mn[g] >> 4) << 6);
    }
}

/* Q4_K / Q5_K: affine groups of 32, 6-bit scales and mins under f16 d/dmin. */
static void quant_kaffine(const float* x, uint8_t* blk, int bits)
{
    const int levels = (1 << bits) - 1;
    float scale[8], mneg[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int g = 0; g < 8; g++) {
        float mn = x[g * 32], mx = x[g * 32];
        for (int i = 1; i < 32; i++) {
            float v = x[g * 32 + i];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mn > 0.0f) mn = 0.0f;
        scale[g] = (mx - mn) / (float)levels;
        mneg[g] = -mn;
        if (scale[g] > max_scale) max_scale = scale[g];
        if (mneg[g] > max_min) max_min = mneg[g];
    }
    uint16_t d16 = gg_f32_to_f16(max_scale / 63.0f), m16 = gg_f32_to_f16(max_min / 63.0f);
    float d = gg_f16_to_f32(d16), dmin = gg_f16_to_f32(m16);
    int sc[8], mn[8];
    for (int g = 0; g < 8; g++) {
        sc[g] = d > 0.0f ? clampi((int)rintf(scale[g] / d), 0, 63) : 0;
        mn[g] = dmin > 0.0f ? clampi((int)rintf(mneg[g] / dmin), 0, 63) : 0;
    }
    wr16(blk, d16);
    wr16(blk + 2, m16);
    pack_kscale_min(sc, mn, blk + 4);
    uint8_t* qh = bits == 5 ? blk + 16 : NULL;
    uint8_t* qs = bits == 5 ? blk + 48 : blk + 16;
    memset(qs, 0, 128);
    if (qh) memset(qh, 0, 32);
    for (int g = 0; g < 8; g++) {
        float dg = d * (float)sc[g];
        float mg = dmin * (float)mn[g];
        for (int i = 0; i < 32; i++) {
            int e = g * 32 + i;
            int q = dg > 0.0f ? clampi((int)rintf((x[e] + mg) / dg), 0, levels) : 0;
            qs[e >> 1] |= (uint8_t)((q & 0xF) << ((e & 1) * 4));
            if (qh) qh[e >> 3] |= (uint8_t)(((q >> 4) & 1) << (e & 7));
        }
    }
}

/* Q6_K: 16 groups of 16 with int8 scales under an f16 d; q - 32 in [-32, 31]. */
static void quant_q6k(const float* x, uint8_t* blk)
{
    float scale[16], max_abs_scale = 0.0f;
    for (int j = 0; j < 16; j++) {
        float vmax = 0.0f, amax = 0.0f;
        for (int i = 0; i < 16; i++) {
            float v = x[j * 16 + i];
            if (fabsf(v) > amax) { amax = fabsf(v); vmax = v; }
        }
        scale[j] = -vmax / 32.0f; /* the extreme element maps to q = -32 */
        if (fabsf(scale[j]) > max_abs_scale) max_abs_scale = fabsf(scale[j]);
    }
    uint16_t d16 = gg_f32_to_f16(max_abs_scale / 127.0f);
    float d = gg_f16_to_f32(d16);
    uint8_t* ql = blk;
    uint8_t* qh = blk + 128;
    int8_t* sc = (int8_t*)(blk + 192);
    memset(blk, 0, 208);
    for (int j = 0; j < 16; j++) {
        int s = d > 0.0f ? clampi((int)rintf(scale[j] / d), -128, 127) : 0;
        sc[j] = (int8_t)s;
        float ds = d * (float)s;
        for (int i = 0; i < 16; i++) {
            int e = j * 16 + i;
            int q = ds != 0.0f ? clampi((int)rintf(x[e] / ds), -32, 31) : 0;
            q += 32;
            ql[e >> 1] |= (uint8_t)((q & 0xF) << ((e & 1) * 4));
            qh[e >> 2] |= (uint8_t)(((q >> 4) & 3) << ((e & 3) * 2));
        }
    }
    wr16(blk + 208, d16);
}

static void quant_q8_0(const float* x, uint8_t* blk)
{
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) if (fabsf(x[i]) > amax) amax = fabsf(x[i]);
    uint16_t d16 = gg_f32_to_f16(amax / 127.0f);
    float d = gg_f16_to_f32(d16);
    wr16(blk, d16);
    for (int i = 0; i < 32; i++) blk[2 + i] = (uint8_t)(int8_t)(d > 0.0f ? clampi((int)rintf(x[i] / d), -127, 127) : 0);
}

static void quant_q4_0(const float* x, uint8_t* blk)
{
    float vmax = 0.0f, amax = 0.0f;
    for (int i = 0; i < 32; i++) if (fabsf(x[i]) > amax) { amax = fabsf(x[i]); vmax = x[i]; }
    uint16_t d16 = gg_f32_to_f16(vmax / -8.0f);
    float d = gg_f16_to_f32(d16);
    wr16(blk, d16);
    for (int j = 0; j < 16; j++) {
        int lo = d != 0.0f ? clampi((int)rintf(x[j] / d) + 8, 0, 15) : 8;
        int hi = d != 0.0f ? clampi((int)rintf(x[j + 16] / d) + 8, 0, 15) : 8;
        blk[2 + j] = (uint8_t)(lo | (hi << 4));
    }
}

static void quant_q8_k(const float* x, uint8_t* blk)
{
    float amax = 0.0f;
    for (int i = 0; i < 256; i++) if (fabsf(x[i]) > amax) amax = fabsf(x[i]);
    float d = amax / 127.0f;
    memcpy(blk, &d, 4);
    int16_t bsums[16];
    for (int j = 0; j < 16; j++) bsums[j] = 0;
    for (int i = 0; i < 256; i++) {
        int q = d > 0.0f ? clampi((int)rintf(x[i] / d), -127, 127) : 0;
        blk[4 + i] = (uint8_t)(int8_t)q;
        bsums[i >> 4] = (int16_t)(bsums[i >> 4] + q);
    }
    memcpy(blk + 260, bsums, 32);
}

static int block_elems(int t)
{
    switch (t) {
    case T_F32: case T_F16: case T_BF16: return 1;
    case T_Q4_0: case T_Q8_0: return 32;
    case T_Q4_K: case T_Q5_K: case T_Q6_K: case T_Q8_K: return 256;
    default: return -1;
    }
}
static int block_bytes(int t)
{
    switch (t) {
    case T_F32: return 4;
    case T_F16: case T_BF16: return 2;
    case T_Q4_0: return 18;
    case T_Q8_0: return 34;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_Q8_K: return 292;
    default: return -1;
    }
}

int64_t gg_tensor_bytes(int t, int64_t n)
{
    int be = block_elems(t), bb = block_bytes(t);
    if (be <= 0 || n % be != 0) return -1;
    return n / be * bb;
}

static void quant_block(int t, const float* x, uint8_t* out)
{
    switch (t) {
    case T_F32: memcpy(out, x, 4); break;
    case T_F16: wr16(out, gg_f32_to_f16(x[0])); break;
    case T_BF16: wr16(out, f32_to_bf16(x[0])); break;
    case T_Q4_0: quant_q4_0(x, out); break;
    case T_Q8_0: quant_q8_0(x, out); break;
    case T_Q4_K: quant_kaffine(x, out, 4); break;
    case T_Q5_K: quant_kaffine(x, out, 5); break;
    case T_Q6_K: quant_q6k(x, out); break;
    case T_Q8_K: quant_q8_k(x, out); break;
    }
}

/* Quantizes n floats into dst (gg_tensor_bytes(t, n) bytes). */
int64_t gg_quantize(int t, const float* src, int64_t n, uint8_t* dst)
{
    int64_t nbytes = gg_tensor_bytes(t, n);
    if (nbytes < 0) return -1;
    int be = block_elems(t), bb = block_bytes(t);
    int64_t nb = n / be;
#pragma omp parallel for schedule(static) num_threads(nthreads())
    for (int64_t b = 0; b < nb; b++) quant_block(t, src + b * be, dst + b * bb);
    return nbytes;
}

/* Draws n values of stream `stream` and quantizes them straight into dst;
 * no float copy of the tensor is held. */
int64_t gg_random_tensor(int t, uint64_t seed, uint64_t stream, int64_t n, float sigma, uint8_t* dst)
{
    int64_t nbytes = gg_tensor_bytes(t, n);
    if (nbytes < 0) return -1;
    int be = block_elems(t), bb = block_bytes(t);
    int64_t nb = n / be;
    uint64_t base = stream_base(seed, stream);
    const int chunk = 256; /* blocks of 1 element (float types) are batched */
    if (be == 1) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
        for (int64_t c = 0; c < (nb + chunk - 1) / chunk; c++) {
            float x;
            int64_t e = (c + 1) * chunk < nb ? (c + 1) * chunk : nb;
            for (int64_t b = c * chunk; b < e; b++) {
                x = normal_at(base, b, sigma);
                quant_block(t, &x, dst + b * bb);
            }
        }
        return nbytes;
    }
#pragma omp parallel for schedule(static) num_threads(nthreads())
    for (int64_t b = 0; b < nb; b++) {
        float x[256];
        for (int i = 0; i < be; i++) x[i] = normal_at(base, b * be + i, sigma);
        quant_block(t, x, dst + b * bb);
    }
    return nbytes;
}

/* Fills an F32 tensor with a constant (norm weights = 1.0). */
void gg_fill_f32(float* dst, int64_t n, float v)
{
    for (int64_t i = 0; i < n; i++) dst[i] = v;
}
