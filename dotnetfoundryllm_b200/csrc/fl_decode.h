/*
 * fl_decode.h — how a repacked unit (fl_layout.h) is read: the A-fragment
 * registers of the int8 MMA and the per-(row, chunk, half) scale pair.
 * Shared by the CUDA kernel and the host emulation so both read the layout
 * the same way.
 *
 * The value encodings are the reference decoder's
 * (src/DotNetFoundryLLM.Quantization/Dequantizer.cs):
 *   Q4_K/Q5_K  v = (d*sc)*q - (dmin*m)      :281-290, :347-364 (DecodeKScaleMin :506-521)
 *   Q6_K       v = (d*sc)*(q-32)            :404-414
 *   Q8_0       v = q*d                      :226-229
 *   Q4_0       v = (q-8)*d                  :178-183
 *   Q8_K       v = q*d                      :451-454
 * written as v = mul*q - sub per (row, chunk, half).
 */
#ifndef FL_DECODE_H
#define FL_DECODE_H

#include <stdint.h>
#include <string.h>

#include "fl_layout.h"

#ifdef __CUDACC__
#include <cuda_fp16.h>
#define FL_HD __host__ __device__ __forceinline__
#else
#define FL_HD static inline
#endif

typedef struct {
    int32_t qs;    /* offset of the quant words */
    int32_t qh;    /* offset of the high-bit words (Q5_K/Q6_K), else -1 */
    int32_t hdr;   /* header bytes at the unit start */
    int32_t unit;  /* unit bytes */
} fl_unit_off;

FL_HD fl_unit_off fl_offsets(int fmt, int expanded)
{
    fl_unit_off o;
    int h = expanded ? FL_EXP_HDR_BYTES : 0;
    switch (fmt) {
    case FL_FMT_Q4K: o.hdr = expanded ? h : 256; o.qh = -1; o.qs = o.hdr; o.unit = o.hdr + 2048; break;
    case FL_FMT_Q5K: o.hdr = expanded ? h : 256; o.qh = o.hdr; o.qs = o.hdr + 512; o.unit = o.hdr + 2560; break;
    case FL_FMT_Q6K: o.hdr = expanded ? h : 288; o.qh = o.hdr; o.qs = o.hdr + 1024; o.unit = o.hdr + 3072; break;
    case FL_FMT_Q8_0: o.hdr = 256; o.qh = -1; o.qs = 256; o.unit = 4352; break;
    case FL_FMT_Q4_0: o.hdr = 256; o.qh = -1; o.qs = 256; o.unit = 2304; break;
    default: /* FL_FMT_Q8K */ o.hdr = expanded ? h : 64; o.qh = -1; o.qs = o.hdr; o.unit = o.hdr + 4096; break;
    }
    return o;
}

FL_HD int fl_fmt_signed(int fmt) { return fmt == FL_FMT_Q8_0 || fmt == FL_FMT_Q8K; }
FL_HD int fl_fmt_nibbles(int fmt) { return fmt == FL_FMT_Q4K || fmt == FL_FMT_Q5K || fmt == FL_FMT_Q6K || fmt == FL_FMT_Q4_0; }

/* Aligned loads (every offset used below is a multiple of the access size). */
FL_HD uint32_t fl_ld32(const uint8_t* p)
{
#ifdef __CUDA_ARCH__
    return *reinterpret_cast<const uint32_t*>(p);
#else
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
#endif
}

FL_HD uint16_t fl_ld16(const uint8_t* p)
{
#ifdef __CUDA_ARCH__
    return *reinterpret_cast<const uint16_t*>(p);
#else
    uint16_t v;
    memcpy(&v, p, 2);
    return v;
#endif
}

FL_HD float fl_ldf(const uint8_t* p)
{
#ifdef __CUDA_ARCH__
    return *reinterpret_cast<const float*>(p);
#else
    float v;
    memcpy(&v, p, 4);
    return v;
#endif
}

/* Moves the bits of `h` selected by `src_bit` (same position in every byte) to
 * the `dst_bit` position of every byte, masked by `mask`. */
FL_HD uint32_t fl_shift_bits(uint32_t h, int src_bit, int dst_bit, uint32_t mask)
{
    return (src_bit <= dst_bit ? (h << (dst_bit - src_bit)) : (h >> (src_bit - dst_bit))) & mask;
}

/* A registers for chunk c (0..7) of a unit, lane l: a[0] = even values of
 * row g, a[1] = even values of row g+8, a[2] = odd values of row g, a[3] = odd
 * values of row g+8 (4 bytes each; u8 or s8 by format). */
FL_HD void fl_unit_afrag(const uint8_t* unit, int fmt, int expanded, int c, int l, uint32_t a[4])
{
    fl_unit_off o = fl_offsets(fmt, expanded);
    int s = c >> 1, jb = (c & 1) * 2; /* words jb (row g) and jb+1 (row g+8) of step s */
    if (fl_fmt_nibbles(fmt)) {
        const uint8_t* w = unit + o.qs + ((s * 32 + l) * 4) * 4;
        uint32_t w0 = fl_ld32(w + 4 * jb), w1 = fl_ld32(w + 4 * (jb + 1));
        uint32_t e0 = w0 & 0x0F0F0F0Fu, o0 = (w0 >> 4) & 0x0F0F0F0Fu;
        uint32_t e1 = w1 & 0x0F0F0F0Fu, o1 = (w1 >> 4) & 0x0F0F0F0Fu;
        if (fmt == FL_FMT_Q5K) {
            /* byte k of H, bit 2j+p = high bit of value 2k+p of word j */
            uint32_t H = fl_ld32(unit + o.qh + (s * 32 + l) * 4);
            e0 |= fl_shift_bits(H, 2 * jb + 0, 4, 0x10101010u);
            o0 |= fl_shift_bits(H, 2 * jb + 1, 4, 0x10101010u);
            e1 |= fl_shift_bits(H, 2 * (jb + 1) + 0, 4, 0x10101010u);
            o1 |= fl_shift_bits(H, 2 * (jb + 1) + 1, 4, 0x10101010u);
        } else if (fmt == FL_FMT_Q6K) {
            /* H_m (m = c&1) covers words 2m (w=0) and 2m+1 (w=1): byte k bits
             * [2(2w+p), 2(2w+p)+1] = high 2 bits of value 2k+p */
            uint32_t H = fl_ld32(unit + o.qh + (s * 32 + l) * 8 + (c & 1) * 4);
            e0 |= fl_shift_bits(H, 0, 4, 0x30303030u);
            o0 |= fl_shift_bits(H, 2, 4, 0x30303030u);
            e1 |= fl_shift_bits(H, 4, 4, 0x30303030u);
            o1 |= fl_shift_bits(H, 6, 4, 0x30303030u);
        }
        a[0] = e0; a[1] = e1; a[2] = o0; a[3] = o1;
    } else {
        /* Q8_0 / Q8_K: [step][half][lane][16 B]; half = c&1 holds words jb, jb+1,
         * each 8 bytes = 4 even values then 4 odd values. */
        const uint8_t* w = unit + o.qs + (((s * 2 + (c & 1)) * 32 + l) * 16);
        a[0] = fl_ld32(w + 0);  /* row g even */
        a[2] = fl_ld32(w + 4);  /* row g odd */
        a[1] = fl_ld32(w + 8);  /* row g+8 even */
        a[3] = fl_ld32(w + 12); /* row g+8 odd */
    }
}

FL_HD float fl_half_to_float(uint16_t h)
{
#ifdef __CUDA_ARCH__
    /* a NaN comes back quiet with its payload, as (float)Half does on the host */
    if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu))
        return __uint_as_float(((uint32_t)(h & 0x8000u) << 16) | 0x7FC00000u | ((uint32_t)(h & 0x3FFu) << 13));
    return __half2float(__ushort_as_half(h));
#else
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
    } else if (exp == 0x1F) out = man ? (sign | 0x7FC00000u | (man << 13)) : (sign | 0x7F800000u);
    else out = sign | ((exp + 112u) << 23) | (man << 13);
    float f;
    memcpy(&f, &out, 4);
    return f;
#endif
}

/* DecodeKScaleMin (Dequantizer.cs:506-521). */
FL_HD void fl_kscale_min(const uint8_t* p, int g, int* sc, int* mn)
{
    if (g < 4) {
        *sc = p[g] & 0x3F;
        *mn = p[g + 4] & 0x3F;
    } else {
        *sc = (p[g + 4] & 0x0F) | ((p[g - 4] >> 6) << 4);
        *mn = (p[g + 4] >> 4) | ((p[g] >> 6) << 4);
    }
}

/* (mul, sub) of row r (0..15), chunk c, half h of a unit. */
FL_HD void fl_unit_scale(const uint8_t* unit, int fmt, int expanded, int r, int c, int h, float* mul, float* sub)
{
    if (expanded) {
        const uint8_t* e = unit + ((r * 8 + c) * 2 + h) * 8;
        *mul = fl_ldf(e);
        *sub = fl_ldf(e + 4);
        return;
    }
    switch (fmt) {
    case FL_FMT_Q4K:
    case FL_FMT_Q5K: {
        const uint8_t* hd = unit + r * 16;
        uint16_t db = fl_ld16(hd), mb = fl_ld16(hd + 2);
        int sc, mn;
        fl_kscale_min(hd + 4, c, &sc, &mn);
        *mul = fl_half_to_float(db) * (float)sc;
        *sub = fl_half_to_float(mb) * (float)mn;
        break;
    }
    case FL_FMT_Q6K: {
        int8_t sc = (int8_t)unit[FL_Q6K_SC + r * 16 + c * 2 + h];
        uint16_t db = fl_ld16(unit + FL_Q6K_D + r * 2);
        float m = fl_half_to_float(db) * (float)sc;
        *mul = m;
        *sub = 32.0f * m;
        break;
    }
    case FL_FMT_Q8_0:
    case FL_FMT_Q4_0: {
        float d = fl_half_to_float(fl_ld16(unit + (r * 8 + c) * 2));
        *mul = d;
        *sub = fmt == FL_FMT_Q4_0 ? 8.0f * d : 0.0f;
        break;
    }
    default: { /* Q8_K */
        float d = fl_ldf(unit + r * 4);
        *mul = d;
        *sub = 0.0f;
        break;
    }
    }
}

#endif
