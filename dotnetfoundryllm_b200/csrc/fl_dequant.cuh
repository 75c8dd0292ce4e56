/*
 * fl_dequant.cuh — element-wise dequantization with the reference decoder's
 * formulas and rounding order (src/DotNetFoundryLLM.Quantization/
 * Dequantizer.cs), bit-exact: explicit _rn intrinsics, no FMA contraction.
 */
#ifndef FL_DEQUANT_CUH
#define FL_DEQUANT_CUH

#include <cuda_fp16.h>
#include <stdint.h>

#include "fl_decode.h"

__device__ __forceinline__ float fl_dq_half(const uint8_t* p) { return fl_half_to_float((uint16_t)(p[0] | (p[1] << 8))); }

/* Dequantizer.cs element formulas with the reference's rounding order
 * (explicit _rn intrinsics: no contraction into FMA). */
__device__ __forceinline__ float fl_dequant_elem(int type, const uint8_t* __restrict__ raw, int64_t f)
{
    switch (type) {
    case FL_T_F32: return __uint_as_float((uint32_t)raw[4 * f] | ((uint32_t)raw[4 * f + 1] << 8) |
                                          ((uint32_t)raw[4 * f + 2] << 16) | ((uint32_t)raw[4 * f + 3] << 24));
    case FL_T_F16: return fl_dq_half(raw + 2 * f);
    case FL_T_BF16: return __uint_as_float(((uint32_t)raw[2 * f] | ((uint32_t)raw[2 * f + 1] << 8)) << 16);
    case FL_T_Q4_0: { /* :178-183 */
        const uint8_t* b = raw + (f / 32) * 18;
        int j = (int)(f % 32);
        int q = j < 16 ? (b[2 + j] & 0x0F) : (b[2 + j - 16] >> 4);
        return __fmul_rn((float)(q - 8), fl_dq_half(b));
    }
    case FL_T_Q8_0: { /* :226-229 */
        const uint8_t* b = raw + (f / 32) * 34;
        return __fmul_rn((float)(int8_t)b[2 + f % 32], fl_dq_half(b));
    }
    case FL_T_Q4_K:
    case FL_T_Q5_K: { /* :268-293, :333-367 */
        const int bb = type == FL_T_Q4_K ? 144 : 176;
        const uint8_t* b = raw + (f / 256) * bb;
        int e = (int)(f % 256);
        int sc, mn;
        fl_kscale_min(b + 4, e / 32, &sc, &mn);
        float dg = __fmul_rn(fl_dq_half(b), (float)sc);
        float mg = __fmul_rn(fl_dq_half(b + 2), (float)mn);
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
        return __fmul_rn(__fmul_rn(fl_dq_half(b + 208), (float)s), (float)q);
    }
    default: { /* FL_T_Q8_K :444-455 */
        const uint8_t* b = raw + (f / 256) * 292;
        float d = __uint_as_float((uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24));
        return __fmul_rn((float)(int8_t)b[4 + f % 256], d);
    }
    }
}

#endif
