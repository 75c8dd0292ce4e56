/*
 * fl_mv_core.cuh — the dequant-matvec building blocks shared by the
 * standalone matvec kernel (fl_matvec.cu) and the persistent token kernel
 * (fl_token.cu): the producer-op prologue, the 3-limb int8 encoding of the
 * input vector, the per-unit int8 tensor-core MMA + scale arithmetic of every
 * quantized format, and the consumer-op epilogues.
 *
 * Reference: LinearProjection over F32 weights
 * (src/DotNetFoundryLLM.Architectures/LlamaForwardPass.cs:237-260) with the
 * weights of src/DotNetFoundryLLM.Quantization/Dequantizer.cs.
 *
 * Values written by an earlier phase of the same kernel are read with
 * ld.global.cg (L2), never through the non-coherent L1.
 */
#ifndef FL_MV_CORE_CUH
#define FL_MV_CORE_CUH

#include <math.h>

#include "fl_decode.h"
#include "fl_dequant.cuh"
#include "fl_device.cuh"
#include "fl_kernels.h"

namespace flcore {

constexpr float kMagic = 12582912.0f; /* 1.5 * 2^23: y + kMagic rounds y to an integer in the low mantissa */
constexpr int kRedSlots = 4;          /* tiles whose cross-warp reduction can be in flight */

__device__ __forceinline__ int seg_of(const FlMvArgs& a, int tile)
{
    int s = 0;
#pragma unroll
    for (int i = 1; i < FL_MV_MAX_SEG; i++)
        if (i < a.n_seg && tile >= a.seg[i].tile0) s = i;
    return s;
}

/* The prologue transform: the op that produced the vector in the reference. */
struct Prolog {
    int mode, K;
    const float *x, *w, *pend, *pw;
    float rms, rms_p;
    __device__ __forceinline__ float resid(int i) const
    {
        /* x' = x + GemmaRmsNorm(pend, pw)  (Gemma2ForwardPass.cs:90-91, 95-96) */
        float pn = __fmul_rn(__fmul_rn(__ldcg(pend + i), rms_p), __fadd_rn(pw[i], 1.0f));
        return __fadd_rn(__ldcg(x + i), pn);
    }
    __device__ __forceinline__ float value(int i) const
    {
        if (i >= K) return 0.0f;
        switch (mode) {
        case FL_IN_PLAIN: return __ldcg(x + i);
        case FL_IN_RMSNORM: return __fmul_rn(__fmul_rn(__ldcg(x + i), rms), w[i]);      /* TensorOperations.cs:49-53 */
        case FL_IN_GEMMA_NORM: return __fmul_rn(__fmul_rn(__ldcg(x + i), rms), __fadd_rn(w[i], 1.0f)); /* :92-101 */
        default: return __fmul_rn(__fmul_rn(resid(i), rms), __fadd_rn(w[i], 1.0f));
        }
    }
};

/* Lane l encodes word (c = l>>2, t = l&3) of k-block kb — the input values
 * kb*256 + 8l .. kb*256 + 8l + 7, given in v — into 3 limbs (B-fragment
 * order), the limb sums of its half-chunk and the float half sums.
 *
 * y = v * inv (|y| <= 127) is rounded once to the 2^-14 grid, Y = rint(y *
 * 2^14) (one FMA against the 1.5 * 2^23 rounding constant; |Y| < 2^22), and
 * Y is cut into X0 * 2^14 + X1 * 2^7 + X2 with X0 in [-127, 127], X1 in
 * [-64, 64], X2 in [-64, 63]: y = X0 + X1/128 + X2/16384 within 2^-15, in
 * integer operations. */
__device__ __forceinline__ void encode_values(const float (&v)[8], int kb, float inv, int lane, uint8_t* xl, short2* xs,
                                              float* xsum)
{
    const int c = lane >> 2, t = lane & 3;
    const int cg = kb * 8 + c;
    const float inv14 = inv * 16384.0f; /* exact: a power-of-two scale */
    int X[3][8];
    float hs = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        hs += v[i];
        const int Y = __float_as_int(fmaf(v[i], inv14, kMagic)) - __float_as_int(kMagic);
        const int x0 = (Y + 8192) >> 14;
        const int r = Y - (x0 << 14);
        const int x1 = (r + 64) >> 7;
        X[0][i] = x0;
        X[1][i] = x1;
        X[2][i] = r - (x1 << 7);
    }
    uint32_t lo[3], hi[3];
    int sl[3];
#pragma unroll
    for (int l = 0; l < 3; l++) {
        /* even values into lo, odd into hi, byte k = value 2k (+1) */
        const uint32_t e01 = __byte_perm((uint32_t)X[l][0], (uint32_t)X[l][2], 0x0040u);
        const uint32_t e23 = __byte_perm((uint32_t)X[l][4], (uint32_t)X[l][6], 0x0040u);
        const uint32_t o01 = __byte_perm((uint32_t)X[l][1], (uint32_t)X[l][3], 0x0040u);
        const uint32_t o23 = __byte_perm((uint32_t)X[l][5], (uint32_t)X[l][7], 0x0040u);
        lo[l] = __byte_perm(e01, e23, 0x5410u);
        hi[l] = __byte_perm(o01, o23, 0x5410u);
        sl[l] = __dp4a((int)lo[l], 0x01010101, __dp4a((int)hi[l], 0x01010101, 0));
    }
#pragma unroll
    for (int l = 0; l < 3; l++)
        *reinterpret_cast<uint2*>(xl + (size_t)cg * FL_XENC_LIMB_BYTES + (l * 4 + t) * 8) = make_uint2(lo[l], hi[l]);
    /* half = words {0,1} or {2,3}: combine with the neighbouring lane */
#pragma unroll
    for (int l = 0; l < 3; l++) sl[l] += __shfl_xor_sync(0xffffffffu, sl[l], 1);
    hs += __shfl_xor_sync(0xffffffffu, hs, 1);
    xs[cg * 4 + t] = (t & 1) ? make_short2((short)sl[2], 0) : make_short2((short)sl[0], (short)sl[1]);
    if ((t & 1) == 0) xsum[cg * 2 + (t >> 1)] = hs;
}

__device__ __forceinline__ void encode_kblock(const Prolog& P, int kb, float inv, int lane, uint8_t* xl, short2* xs,
                                              float* xsum)
{
    float v[8];
    const int base = kb * 256 + lane * 8;
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = P.value(base + i);
    encode_values(v, kb, inv, lane, xl, xs, xsum);
}

struct Acc {
    float res0, res1; /* limb-weighted sums of rows g, g+8 (scaled by W_t * s at the end) */
    float m0, m1;     /* absolute-valued min/offset terms */
};

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int k) { return (w >> (8 * k)) & 0xFFu; }
__device__ __forceinline__ int sbyte_of(uint32_t w, int k) { return (int)(int8_t)((w >> (8 * k)) & 0xFFu); }
__device__ __forceinline__ float h2f(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)bits16)); }

/* One unit (16 rows x 256 columns) in shared memory.  Its bytes are first
 * copied to registers and `release()` is called — the slot may then be
 * refilled while this unit is computed — then come the 8 int8 MMAs and the
 * scale arithmetic of the format.  (With expanded headers the per-chunk float
 * pairs are read as the chunks go, so the slot is released at the end.)
 *
 * bp: this lane's B fragment of chunk 0 of the unit's k-block (chunk c at
 * bp + c * FL_XENC_LIMB_BYTES), or a zero area for lanes whose column is not
 * theirs. */
template <int FMT, bool EXP, typename Release>
__device__ __forceinline__ void process_unit(const uint8_t* __restrict__ u, int kb, const uint8_t* __restrict__ bp,
                                             const short2* __restrict__ xs, const float* __restrict__ xsum, int lane,
                                             Acc& A, Release&& release)
{
    const int g = lane >> 2, t = lane & 3, h = t >> 1;
    constexpr bool NIB = FMT == FL_FMT_Q4K || FMT == FL_FMT_Q5K || FMT == FL_FMT_Q6K || FMT == FL_FMT_Q4_0;
    constexpr bool SIGNED = FMT == FL_FMT_Q8_0 || FMT == FL_FMT_Q8K;
    constexpr int NW4 = NIB ? 4 : 8; /* uint4 words of quants per lane */
    const fl_unit_off o = fl_offsets(FMT, EXP);
    const short2* xsk = xs + kb * 8 * 4 + t;

    /* ── stage the unit in registers ── */
    uint4 W[NW4];
    uint32_t H5[4] = {0, 0, 0, 0};
    uint2 H6[4] = {make_uint2(0, 0), make_uint2(0, 0), make_uint2(0, 0), make_uint2(0, 0)};
#pragma unroll
    for (int i = 0; i < NW4; i++) W[i] = *reinterpret_cast<const uint4*>(u + o.qs + (i * 32 + lane) * 16);
    if constexpr (FMT == FL_FMT_Q5K) {
#pragma unroll
        for (int s = 0; s < 4; s++) H5[s] = *reinterpret_cast<const uint32_t*>(u + o.qh + (s * 32 + lane) * 4);
    }
    if constexpr (FMT == FL_FMT_Q6K) {
#pragma unroll
        for (int s = 0; s < 4; s++) H6[s] = *reinterpret_cast<const uint2*>(u + o.qh + (s * 32 + lane) * 8);
    }
    uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0; /* header words of rows g, g+8 */
    float dd0 = 0.0f, dd1 = 0.0f;               /* Q6_K / Q8_K super-block scales */
    if constexpr (!EXP) {
        if constexpr (FMT == FL_FMT_Q6K) {
            h0 = *reinterpret_cast<const uint4*>(u + FL_Q6K_SC + g * 16);
            h1 = *reinterpret_cast<const uint4*>(u + FL_Q6K_SC + (g + 8) * 16);
            dd0 = h2f(*reinterpret_cast<const uint16_t*>(u + FL_Q6K_D + g * 2));
            dd1 = h2f(*reinterpret_cast<const uint16_t*>(u + FL_Q6K_D + (g + 8) * 2));
        } else if constexpr (FMT == FL_FMT_Q8K) {
            dd0 = *reinterpret_cast<const float*>(u + g * 4);
            dd1 = *reinterpret_cast<const float*>(u + (g + 8) * 4);
        } else {
            h0 = *reinterpret_cast<const uint4*>(u + g * 16);
            h1 = *reinterpret_cast<const uint4*>(u + (g + 8) * 16);
        }
        release();
    }

    /* ── per-unit scale state ── */
    uint32_t scw0[4] = {0, 0, 0, 0}, scw1[4] = {0, 0, 0, 0};
    if constexpr (!EXP) {
        if constexpr (FMT == FL_FMT_Q4K || FMT == FL_FMT_Q5K) {
            /* packed DecodeKScaleMin: 4 scales per word */
            scw0[0] = h0.y & 0x3F3F3F3Fu;
            scw0[1] = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
            scw0[2] = h0.z & 0x3F3F3F3Fu;
            scw0[3] = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
            scw1[0] = h1.y & 0x3F3F3F3Fu;
            scw1[1] = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
            scw1[2] = h1.z & 0x3F3F3F3Fu;
            scw1[3] = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
            /* min term: this lane takes chunks 2t and 2t+1 of both rows */
            const float4 sx = *reinterpret_cast<const float4*>(xsum + (kb * 8 + 2 * t) * 2);
            const float sa = sx.x + sx.y, sb = sx.z + sx.w;
            const uint32_t mw0 = t < 2 ? scw0[2] : scw0[3], mw1 = t < 2 ? scw1[2] : scw1[3];
            const int ka = 2 * (t & 1);
            const float M0 = fmaf((float)byte_of(mw0, ka), sa, (float)byte_of(mw0, ka + 1) * sb);
            const float M1 = fmaf((float)byte_of(mw1, ka), sa, (float)byte_of(mw1, ka + 1) * sb);
            A.m0 = fmaf(h2f(h0.x >> 16), M0, A.m0);
            A.m1 = fmaf(h2f(h1.x >> 16), M1, A.m1);
        } else {
            scw0[0] = h0.x; scw0[1] = h0.y; scw0[2] = h0.z; scw0[3] = h0.w;
            scw1[0] = h1.x; scw1[1] = h1.y; scw1[2] = h1.z; scw1[3] = h1.w;
        }
    }

    /* every B fragment (and Q6_K/Q4_0 limb sum) of the unit up front, so the
     * 8 MMAs do not each wait on their own shared-memory load */
    uint2 bf[8];
#pragma unroll
    for (int c = 0; c < 8; c++) bf[c] = *reinterpret_cast<const uint2*>(bp + c * FL_XENC_LIMB_BYTES);
    short2 lsum[8];
    if constexpr ((FMT == FL_FMT_Q6K || FMT == FL_FMT_Q4_0) && !EXP) {
#pragma unroll
        for (int c = 0; c < 8; c++) lsum[c] = xsk[c * 4];
    }

    int ia0 = 0, ia1 = 0, ib0 = 0, ib1 = 0; /* int32 accumulators: rows g, g+8 x limb pair */
#pragma unroll
    for (int s = 0; s < 4; s++) {
#pragma unroll
        for (int cc = 0; cc < 2; cc++) {
            const int c = 2 * s + cc;
            uint32_t a[4];
            if constexpr (NIB) {
                const uint4 Ws = W[s];
                const uint32_t wg = cc ? Ws.z : Ws.x, wg8 = cc ? Ws.w : Ws.y;
                a[0] = wg & 0x0F0F0F0Fu;
                a[2] = (wg >> 4) & 0x0F0F0F0Fu;
                a[1] = wg8 & 0x0F0F0F0Fu;
                a[3] = (wg8 >> 4) & 0x0F0F0F0Fu;
                if constexpr (FMT == FL_FMT_Q5K) {
                    const int j0 = 2 * cc, j1 = 2 * cc + 1; /* words of rows g, g+8 */
                    a[0] |= fl_shift_bits(H5[s], 2 * j0, 4, 0x10101010u);
                    a[2] |= fl_shift_bits(H5[s], 2 * j0 + 1, 4, 0x10101010u);
                    a[1] |= fl_shift_bits(H5[s], 2 * j1, 4, 0x10101010u);
                    a[3] |= fl_shift_bits(H5[s], 2 * j1 + 1, 4, 0x10101010u);
                }
                if constexpr (FMT == FL_FMT_Q6K) {
                    const uint32_t Hc = cc ? H6[s].y : H6[s].x;
                    a[0] |= (Hc << 4) & 0x30303030u;
                    a[2] |= (Hc << 2) & 0x30303030u;
                    a[1] |= Hc & 0x30303030u;
                    a[3] |= (Hc >> 2) & 0x30303030u;
                }
            } else {
                const uint4 V = W[c];
                a[0] = V.x;
                a[2] = V.y;
                a[1] = V.z;
                a[3] = V.w;
            }
            int d[4];
            fl_mma_i8<SIGNED>(d, a, bf[c].x, bf[c].y);
            if constexpr ((FMT == FL_FMT_Q6K || FMT == FL_FMT_Q4_0) && !EXP) {
                /* (q - off) x = q x - off * sum(x): integer correction per limb
                 * (expanded headers carry the offset in `sub` instead) */
                constexpr int off = FMT == FL_FMT_Q6K ? 32 : 8;
                const short2 S = lsum[c];
                d[0] -= off * S.x;
                d[1] -= off * S.y;
                d[2] -= off * S.x;
                d[3] -= off * S.y;
            }
            if constexpr (EXP) {
                /* straddling rows: per-chunk float (mul, sub) */
                const float2 e0 = *reinterpret_cast<const float2*>(u + ((g * 8 + c) * 2 + h) * 8);
                const float2 e1 = *reinterpret_cast<const float2*>(u + (((g + 8) * 8 + c) * 2 + h) * 8);
                const float p0 = fmaf((float)d[1], 1.0f / 128.0f, (float)d[0]);
                const float p1 = fmaf((float)d[3], 1.0f / 128.0f, (float)d[2]);
                A.res0 = fmaf(e0.x, p0, A.res0);
                A.res1 = fmaf(e1.x, p1, A.res1);
                if ((t & 1) == 0) {
                    const float sxh = xsum[(kb * 8 + c) * 2 + h];
                    A.m0 = fmaf(e0.y, sxh, A.m0);
                    A.m1 = fmaf(e1.y, sxh, A.m1);
                }
            } else if constexpr (FMT == FL_FMT_Q4K || FMT == FL_FMT_Q5K) {
                const int sg = (int)byte_of(c < 4 ? scw0[0] : scw0[1], c & 3);
                const int sg8 = (int)byte_of(c < 4 ? scw1[0] : scw1[1], c & 3);
                ia0 += sg * d[0];
                ia1 += sg * d[1];
                ib0 += sg8 * d[2];
                ib1 += sg8 * d[3];
            } else if constexpr (FMT == FL_FMT_Q6K) {
                /* int8 scale of (chunk c, half h) = byte 2c+h of the row's 16 */
                const int k = 2 * c + h;
                const int sg = sbyte_of(scw0[k >> 2], k & 3), sg8 = sbyte_of(scw1[k >> 2], k & 3);
                ia0 += sg * d[0];
                ia1 += sg * d[1];
                ib0 += sg8 * d[2];
                ib1 += sg8 * d[3];
            } else if constexpr (FMT == FL_FMT_Q8K) {
                ia0 += d[0];
                ia1 += d[1];
                ib0 += d[2];
                ib1 += d[3];
            } else { /* Q8_0 / Q4_0: f16 d per chunk */
                const float dg = h2f((scw0[c >> 1] >> (16 * (c & 1))) & 0xFFFFu);
                const float dg8 = h2f((scw1[c >> 1] >> (16 * (c & 1))) & 0xFFFFu);
                A.res0 = fmaf(dg, fmaf((float)d[1], 1.0f / 128.0f, (float)d[0]), A.res0);
                A.res1 = fmaf(dg8, fmaf((float)d[3], 1.0f / 128.0f, (float)d[2]), A.res1);
            }
        }
    }
    if constexpr (!EXP) {
        if constexpr (FMT == FL_FMT_Q4K || FMT == FL_FMT_Q5K) {
            A.res0 = fmaf(h2f(h0.x & 0xFFFFu), fmaf((float)ia1, 1.0f / 128.0f, (float)ia0), A.res0);
            A.res1 = fmaf(h2f(h1.x & 0xFFFFu), fmaf((float)ib1, 1.0f / 128.0f, (float)ib0), A.res1);
        } else if constexpr (FMT == FL_FMT_Q6K || FMT == FL_FMT_Q8K) {
            A.res0 = fmaf(dd0, fmaf((float)ia1, 1.0f / 128.0f, (float)ia0), A.res0);
            A.res1 = fmaf(dd1, fmaf((float)ib1, 1.0f / 128.0f, (float)ib0), A.res1);
        }
    } else {
        release();
    }
}

struct NoRelease {
    __device__ __forceinline__ void operator()() const {}
};

/* The unit's B-fragment base for this lane (see process_unit). */
__device__ __forceinline__ const uint8_t* unit_bptr(const uint8_t* bptr, bool bval, const uint8_t* zero, int kb)
{
    return bval ? bptr + (size_t)kb * 8 * FL_XENC_LIMB_BYTES : zero;
}

__device__ __forceinline__ void process_any(int fmt, int expanded, const uint8_t* u, int kb, const uint8_t* bp,
                                            const short2* xs, const float* xsum, int lane, Acc& A)
{
    NoRelease r;
    if (expanded) {
        switch (fmt) {
        case FL_FMT_Q4K: process_unit<FL_FMT_Q4K, true>(u, kb, bp, xs, xsum, lane, A, r); break;
        case FL_FMT_Q5K: process_unit<FL_FMT_Q5K, true>(u, kb, bp, xs, xsum, lane, A, r); break;
        case FL_FMT_Q6K: process_unit<FL_FMT_Q6K, true>(u, kb, bp, xs, xsum, lane, A, r); break;
        default: process_unit<FL_FMT_Q8K, true>(u, kb, bp, xs, xsum, lane, A, r); break;
        }
        return;
    }
    switch (fmt) {
    case FL_FMT_Q4K: process_unit<FL_FMT_Q4K, false>(u, kb, bp, xs, xsum, lane, A, r); break;
    case FL_FMT_Q5K: process_unit<FL_FMT_Q5K, false>(u, kb, bp, xs, xsum, lane, A, r); break;
    case FL_FMT_Q6K: process_unit<FL_FMT_Q6K, false>(u, kb, bp, xs, xsum, lane, A, r); break;
    case FL_FMT_Q8_0: process_unit<FL_FMT_Q8_0, false>(u, kb, bp, xs, xsum, lane, A, r); break;
    case FL_FMT_Q4_0: process_unit<FL_FMT_Q4_0, false>(u, kb, bp, xs, xsum, lane, A, r); break;
    default: process_unit<FL_FMT_Q8K, false>(u, kb, bp, xs, xsum, lane, A, r); break;
    }
}

__device__ __forceinline__ float silu_ref(float g)
{
    /* TensorOperations.Silu: x * sigmoid(x), sigmoid = 1 / (1 + exp(-x)) */
    float sig = 1.0f / __fadd_rn(1.0f, expf(-g));
    return __fmul_rn(g, sig);
}

__device__ __forceinline__ float gelu_ref(float v)
{
    /* TensorOperations.Gelu (TensorOperations.cs:110-117), same evaluation order */
    float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
    float inner = __fmul_rn(0.7978845608f, __fadd_rn(v, cube));
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
}

/* The operand an epilogue reads from memory for lane r's row of a tile: the
 * residual row (FL_EPI_RESID) or the RoPE (cos, sin) pair of a q or k row
 * (FL_EPI_QKV).  A warp loads it for its first and last tile before their
 * units, so the epilogue does not wait on memory after them. */
__device__ __forceinline__ float2 epilogue_operand(const FlMvArgs& a, int tile, int lane, int pos)
{
    const int si = seg_of(a, tile);
    const FlMvSeg& sg = a.seg[si];
    const int row_local = (tile - sg.tile0) * 16 + (lane & 15);
    if (lane >= 16 || row_local >= sg.rows) return make_float2(0.0f, 0.0f);
    if (a.epi == FL_EPI_RESID) return make_float2(__ldcg(a.y + sg.tile0 * 16 + row_local), 0.0f);
    if (a.epi == FL_EPI_QKV && si < 2) {
        const int d = row_local % a.head_dim, half = a.head_dim >> 1;
        return *reinterpret_cast<const float2*>(a.rope_cs + ((size_t)pos * half + (d >> 1)) * 2);
    }
    return make_float2(0.0f, 0.0f);
}

/* Runs in the warp that completed the tile; lane r < 16 holds row r in v.
 * All 32 lanes call it (shuffles).  With has_pre, `pre` is the tile's
 * epilogue_operand. */
template <int EPI>
__device__ __forceinline__ void epilogue(const FlMvArgs& a, const FlMvSeg& sg, int si, int tile, int lane, float v,
                                         int pos, float& best_v, int& best_i, float2 pre = make_float2(0.0f, 0.0f),
                                         bool has_pre = false, uint32_t tag = 0)
{
    const int r = lane & 15;
    const bool act = lane < 16;
    const int row_local = (tile - sg.tile0) * 16 + r;
    const bool in_seg = act && row_local < sg.rows;
    if constexpr (EPI == FL_EPI_STORE || EPI == FL_EPI_RESID) {
        if (in_seg) {
            const int row = sg.tile0 * 16 + row_local;
            if (EPI == FL_EPI_STORE) {
                const float o = sg.bias ? __fadd_rn(v, sg.bias[row_local]) : v;
                if (a.tp_n > 0) {
                    /* a row-parallel projection's (partial) row, with the
                     * exchange tag, into this rank's receive slot of every
                     * rank: one 8-byte store each (NVLink for the peers), so
                     * a reader sees the value and its tag together */
                    const unsigned long long word = (unsigned long long)__float_as_uint(o) |
                                                    ((unsigned long long)tag << 32);
                    for (int q = 0; q < a.tp_n; q++)
                        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(
                                         reinterpret_cast<unsigned long long*>(a.tp_out[q]) + row),
                                     "l"(word)
                                     : "memory");
                } else {
                    a.y[row] = o;
                }
            } else {
                a.y[row] = __fadd_rn(has_pre ? pre.x : __ldcg(a.y + row), v);
            }
        }
    } else if constexpr (EPI == FL_EPI_QKV) {
        if (sg.bias && in_seg) v = __fadd_rn(v, sg.bias[row_local]);
        const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
        if (in_seg) {
            if (si < 2) {
                /* TensorOperations.ApplyRope (TensorOperations.cs:250-260) with the
                 * host-computed cos/sin of pos*invFreq[i] */
                const int d = row_local % a.head_dim, i = d >> 1, half = a.head_dim >> 1;
                const float2 cs = has_pre ? pre : *reinterpret_cast<const float2*>(a.rope_cs + ((size_t)pos * half + i) * 2);
                float o;
                if ((d & 1) == 0) o = __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(partner, cs.y));
                else o = __fadd_rn(__fmul_rn(partner, cs.y), __fmul_rn(v, cs.x));
                if (si == 0) a.q_out[row_local] = o;
                else a.k_cache[(size_t)pos * a.kv_rows + row_local] = o;
            } else {
                a.v_cache[(size_t)pos * a.kv_rows + row_local] = v;
            }
        }
    } else if constexpr (EPI == FL_EPI_GLU) {
        /* tile rows 0..7 are gate rows 8*tile.., rows 8..15 the matching up rows */
        const float up = __shfl_sync(0xffffffffu, v, (lane + 8) & 31);
        float actv = 0.0f;
        const int j = tile * 8 + r;
        if (lane < 8 && j < a.rows_total) {
            float gv = a.act_gelu ? gelu_ref(v) : silu_ref(v);
            actv = __fmul_rn(gv, up);
            a.act_out[j] = actv;
        }
        float m = fl_warp_max(fabsf(actv));
        if (lane == 0) atomicMax(reinterpret_cast<int*>(a.act_absmax), __float_as_int(m));
    } else { /* FL_EPI_LOGITS */
        float val = v;
        int idx = 0x7fffffff;
        const int row = sg.tile0 * 16 + row_local + a.tp_row0;
        if (in_seg) {
            if (a.softcap > 0.0f) {
                /* TensorOperations.SoftCap: x*(1/cap) -> tanh -> *cap */
                float inv = 1.0f / a.softcap;
                val = __fmul_rn(tanhf(__fmul_rn(val, inv)), a.softcap);
            }
            if (a.tp_n > 0) {
                for (int q = 0; q < a.tp_n; q++) a.tp_out[q][row] = val; /* full logits on every rank */
            } else {
                a.y[row] = val;
            }
            idx = row;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, val, o);
            int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (oi != 0x7fffffff && (idx == 0x7fffffff || fl_argmax_better(ov, oi, val, idx))) {
                val = ov;
                idx = oi;
            }
        }
        if (idx != 0x7fffffff && (best_i == 0x7fffffff || fl_argmax_better(val, idx, best_v, best_i))) {
            best_v = val;
            best_i = idx;
        }
    }
}

/* Bounded wait until a reduction slot is free again (done[slot] == gen). */
__device__ __forceinline__ void wait_slot(volatile int* done, int gen, int* err)
{
    if (*done >= gen) return;
    for (uint32_t it = 0; it < (1u << 24); it++) {
        if (*done >= gen) return;
        __nanosleep(32);
    }
    if (err) atomicExch(err, FL_DEV_ERR_TIMEOUT);
}

/* Runtime-dispatched epilogue (the persistent kernel mixes epilogues). */
__device__ __forceinline__ void epilogue_any(const FlMvArgs& a, const FlMvSeg& sg, int si, int tile, int lane, float v,
                                             int pos, float& best_v, int& best_i,
                                             float2 pre = make_float2(0.0f, 0.0f), bool has_pre = false,
                                             uint32_t tag = 0)
{
    switch (a.epi) {
    case FL_EPI_STORE: epilogue<FL_EPI_STORE>(a, sg, si, tile, lane, v, pos, best_v, best_i, pre, false, tag); break;
    case FL_EPI_RESID: epilogue<FL_EPI_RESID>(a, sg, si, tile, lane, v, pos, best_v, best_i, pre, has_pre); break;
    case FL_EPI_QKV: epilogue<FL_EPI_QKV>(a, sg, si, tile, lane, v, pos, best_v, best_i, pre, has_pre); break;
    case FL_EPI_GLU: epilogue<FL_EPI_GLU>(a, sg, si, tile, lane, v, pos, best_v, best_i); break;
    default: epilogue<FL_EPI_LOGITS>(a, sg, si, tile, lane, v, pos, best_v, best_i); break;
    }
}

} // namespace flcore

#endif
