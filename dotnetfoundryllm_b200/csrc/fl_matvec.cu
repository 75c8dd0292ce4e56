/*
 * fl_matvec.cu — fused dequant-matvec for the decode step, sm_100a.
 *
 * Replaces LinearProjection over dequantized F32 weights
 * (src/DotNetFoundryLLM.Architectures/LlamaForwardPass.cs:237-260) and the
 * elementwise op on either side of it.  The weights stay in their GGUF bits
 * (repacked, fl_layout.h); nothing is expanded to F32 in HBM.
 *
 * Per launch:
 *  - grid = min(#tiles, #SMs), 8 warps per CTA.  CTA b owns tiles b, b+G, ...;
 *    warp w owns k-blocks w, w+8, ... of each of them.
 *  - every warp streams its own units (16 rows x 256 columns) HBM → shared
 *    memory with 1-D bulk async copies into a private ring of mbarrier slots.
 *    The first slots are requested before griddepcontrol.wait, so the weight
 *    stream of this kernel overlaps the tail of the previous one.
 *  - the input vector is encoded once per CTA into 3 int8 limbs
 *    (x ≈ s*(X0 + X1/128 + X2/16384), s = max|x|/127): the weights stay
 *    integers (4/5/6/8-bit levels), so each (16 rows x 32 values) chunk is one
 *    m16n8k32 int8 tensor-core MMA whose 8 columns are (limb, half-chunk)
 *    pairs; products are exact integers.
 *  - the per-(row, chunk, half) scale pair (mul, sub) of the reference formula
 *    v = mul*q - sub turns the integer sums into F32 partial sums.
 *  - the prologue applies the producer op (RmsNorm / GemmaRmsNorm / residual
 *    post-norm) and the epilogue the consumer op (residual add, RoPE + KV
 *    append, SiLU/GELU gate, logits softcap + argmax), so the decode step has
 *    one launch per projection group.
 */
#include <math.h>

#include "fl_decode.h"
#include "fl_device.cuh"
#include "fl_kernels.h"

namespace {

constexpr int kStabStride = 18; /* float2 per row in the scale table: 16 used + pad (144 B, bank-conflict free) */
constexpr float kMagic = 12582912.0f; /* 1.5 * 2^23: x + kMagic rounds x to an integer in the low mantissa */

__device__ __forceinline__ int seg_of(const FlMvArgs& a, int tile)
{
    int s = 0;
#pragma unroll
    for (int i = 1; i < FL_MV_MAX_SEG; i++)
        if (i < a.n_seg && tile >= a.seg[i].tile0) s = i;
    return s;
}

/* Encodes 8 consecutive values (one "word" t of chunk c) into the 3 limbs,
 * B-fragment order: per limb 4 bytes of even values then 4 of odd values. */
__device__ __forceinline__ void encode_word(const float (&v)[8], float inv, uint8_t* chunk, int t)
{
    uint32_t lo[3] = {0, 0, 0}, hi[3] = {0, 0, 0};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float y = __fmul_rn(v[i], inv);
#pragma unroll
        for (int l = 0; l < 3; l++) {
            float tq = __fadd_rn(y, kMagic);
            float q = __fsub_rn(tq, kMagic);
            uint32_t byte = __float_as_uint(tq) & 0xFFu;
            if (i & 1) hi[l] |= byte << (8 * (i >> 1));
            else lo[l] |= byte << (8 * (i >> 1));
            y = __fmul_rn(__fsub_rn(y, q), 128.0f);
        }
    }
#pragma unroll
    for (int l = 0; l < 3; l++) *reinterpret_cast<uint2*>(chunk + (l * 4 + t) * 8) = make_uint2(lo[l], hi[l]);
}

/* The 8 input values of word w (chunk w>>2, sub-word w&3) after the prologue
 * transform; values past K are zero. */
struct Prolog {
    int mode, K;
    const float *x, *w, *pend, *pw;
    float rms, rms_p;
    __device__ __forceinline__ float resid(int i) const
    {
        /* x' = x + GemmaRmsNorm(pend, pw) */
        float pn = __fmul_rn(__fmul_rn(pend[i], rms_p), __fadd_rn(pw[i], 1.0f));
        return __fadd_rn(x[i], pn);
    }
    __device__ __forceinline__ float value(int i) const
    {
        switch (mode) {
        case FL_IN_PLAIN: return x[i];
        case FL_IN_RMSNORM: return __fmul_rn(__fmul_rn(x[i], rms), w[i]);
        case FL_IN_GEMMA_NORM: return __fmul_rn(__fmul_rn(x[i], rms), __fadd_rn(w[i], 1.0f));
        default: return __fmul_rn(__fmul_rn(resid(i), rms), __fadd_rn(w[i], 1.0f));
        }
    }
};

template <int FMT>
__device__ __forceinline__ void process_unit(const uint8_t* __restrict__ u, int expanded, int kb,
                                             const uint8_t* __restrict__ xl, const float* __restrict__ sxf,
                                             float2* __restrict__ stab, int lane, float& acc0, float& acc1,
                                             float& min0, float& min1)
{
    const int g = lane >> 2, t = lane & 3, h = t >> 1;
    {
        /* scale table: lane L decodes row L>>1, chunks 4*(L&1)..+3, both halves */
        const int r = lane >> 1, c0 = (lane & 1) * 4;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            float m0, s0, m1, s1;
            fl_unit_scale(u, FMT, expanded, r, c0 + c, 0, &m0, &s0);
            fl_unit_scale(u, FMT, expanded, r, c0 + c, 1, &m1, &s1);
            *reinterpret_cast<float4*>(&stab[r * kStabStride + (c0 + c) * 2]) = make_float4(m0, s0, m1, s1);
        }
    }
    __syncwarp();
    const int limb = g & 3;
    const bool bval = (limb < 3) && ((g >> 2) == h);
#pragma unroll
    for (int c = 0; c < 8; c++) {
        uint32_t af[4];
        fl_unit_afrag(u, FMT, expanded, c, lane, af);
        const int cg = kb * 8 + c;
        uint2 b = make_uint2(0u, 0u);
        if (bval) b = *reinterpret_cast<const uint2*>(xl + cg * FL_XENC_LIMB_BYTES + (limb * 4 + t) * 8);
        int d[4];
        fl_mma_i8<FMT == FL_FMT_Q8_0 || FMT == FL_FMT_Q8K>(d, af, b.x, b.y);
        const int i0 = d[0] * 128 + d[1], i1 = d[2] * 128 + d[3];
        const float2 m0 = stab[g * kStabStride + c * 2 + h];
        const float2 m1 = stab[(g + 8) * kStabStride + c * 2 + h];
        const float sv = sxf[cg * 4 + t];
        acc0 = fmaf((float)i0, m0.x, acc0);
        acc1 = fmaf((float)i1, m1.x, acc1);
        min0 = fmaf(m0.y, sv, min0);
        min1 = fmaf(m1.y, sv, min1);
    }
}

__device__ __forceinline__ void process_any(int fmt, const uint8_t* u, int expanded, int kb, const uint8_t* xl,
                                            const float* sxf, float2* stab, int lane, float& a0, float& a1,
                                            float& m0, float& m1)
{
    switch (fmt) {
    case FL_FMT_Q4K: process_unit<FL_FMT_Q4K>(u, expanded, kb, xl, sxf, stab, lane, a0, a1, m0, m1); break;
    case FL_FMT_Q5K: process_unit<FL_FMT_Q5K>(u, expanded, kb, xl, sxf, stab, lane, a0, a1, m0, m1); break;
    case FL_FMT_Q6K: process_unit<FL_FMT_Q6K>(u, expanded, kb, xl, sxf, stab, lane, a0, a1, m0, m1); break;
    case FL_FMT_Q8_0: process_unit<FL_FMT_Q8_0>(u, 0, kb, xl, sxf, stab, lane, a0, a1, m0, m1); break;
    case FL_FMT_Q4_0: process_unit<FL_FMT_Q4_0>(u, 0, kb, xl, sxf, stab, lane, a0, a1, m0, m1); break;
    default: process_unit<FL_FMT_Q8K>(u, expanded, kb, xl, sxf, stab, lane, a0, a1, m0, m1); break;
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

/* Runs in warp 0 after the cross-warp reduction; lane r < 16 holds row r of
 * the tile in v.  All 32 lanes call it (shuffles). */
template <int EPI>
__device__ __forceinline__ void epilogue(const FlMvArgs& a, const FlMvSeg& sg, int si, int tile, int lane, float v,
                                         float& best_v, int& best_i)
{
    const int r = lane & 15;
    const bool act = lane < 16;
    const int row_local = (tile - sg.tile0) * 16 + r;
    const bool in_seg = act && row_local < sg.rows;
    if constexpr (EPI == FL_EPI_STORE || EPI == FL_EPI_RESID) {
        if (in_seg) {
            const int row = sg.tile0 * 16 + row_local;
            float b = sg.bias ? sg.bias[row_local] : 0.0f;
            if (EPI == FL_EPI_STORE) a.y[row] = sg.bias ? __fadd_rn(v, b) : v;
            else a.y[row] = __fadd_rn(a.y[row], v);
        }
    } else if constexpr (EPI == FL_EPI_QKV) {
        if (sg.bias && in_seg) v = __fadd_rn(v, sg.bias[row_local]);
        const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
        const int pos = *a.pos;
        if (in_seg) {
            if (si < 2) {
                /* TensorOperations.ApplyRope (TensorOperations.cs:250-260) with the
                 * host-computed cos/sin of pos*invFreq[i] */
                const int d = row_local % a.head_dim, i = d >> 1, half = a.head_dim >> 1;
                const float2 cs = *reinterpret_cast<const float2*>(a.rope_cs + ((size_t)pos * half + i) * 2);
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
        const int row = sg.tile0 * 16 + row_local;
        if (in_seg) {
            if (a.softcap > 0.0f) {
                /* TensorOperations.SoftCap: x*(1/cap) -> tanh -> *cap */
                float inv = 1.0f / a.softcap;
                val = __fmul_rn(tanhf(__fmul_rn(val, inv)), a.softcap);
            }
            a.y[row] = val;
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

template <int EPI>
__global__ void __launch_bounds__(FL_MV_THREADS, 1) fl_mv_kernel(const __grid_constant__ FlMvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_scale;
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t = lane & 3;
    const int n_chunks = a.n_kb * 8;
    uint8_t* xl = smem;
    float* sxf = reinterpret_cast<float*>(smem + (size_t)n_chunks * FL_XENC_LIMB_BYTES);
    size_t off = ((size_t)n_chunks * (FL_XENC_LIMB_BYTES + FL_XENC_SX_BYTES) + 127) & ~(size_t)127;
    uint8_t* ring = smem + off;
    off += (size_t)FL_MV_WARPS * a.n_slots * a.slot_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + off);
    off += (size_t)FL_MV_WARPS * a.n_slots * 8;
    off = (off + 15) & ~(size_t)15;
    float2* stab = reinterpret_cast<float2*>(smem + off);
    off += (size_t)FL_MV_WARPS * 16 * kStabStride * 8;
    float* red = reinterpret_cast<float*>(smem + off);
    off += 2 * FL_MV_WARPS * 16 * 4;
    float* scratch = reinterpret_cast<float*>(smem + off);

    const int G = gridDim.x;
    const int my_tiles = a.n_tiles > (int)blockIdx.x ? (a.n_tiles - (int)blockIdx.x + G - 1) / G : 0;
    const int upt = warp < a.n_kb ? (a.n_kb - warp + 7) / 8 : 0;
    const int total = my_tiles * upt;
    uint8_t* wring = ring + (size_t)warp * a.n_slots * a.slot_bytes;
    uint64_t* wbar = bars + warp * a.n_slots;
    float2* wstab = stab + warp * 16 * kStabStride;

    if (lane == 0)
        for (int i = 0; i < a.n_slots; i++) fl_mbar_init(&wbar[i], 1);
    if (tid == 0) s_abort = 0;
    fl_fence_mbar_init();
    __syncthreads();

    auto issue = [&](int j) {
        const int tile = (int)blockIdx.x + (j / upt) * G;
        const int kb = warp + 8 * (j % upt);
        const FlMvSeg& sg = a.seg[seg_of(a, tile)];
        const uint8_t* src = sg.w + ((size_t)(tile - sg.tile0) * a.n_kb + kb) * sg.unit_bytes;
        const int slot = j % a.n_slots;
        fl_mbar_expect_tx(&wbar[slot], (uint32_t)sg.unit_bytes);
        fl_bulk_g2s(wring + (size_t)slot * a.slot_bytes, src, (uint32_t)sg.unit_bytes, &wbar[slot]);
    };

    /* weights do not depend on the previous kernel: start streaming them now */
    if (lane == 0)
        for (int j = 0; j < total && j < a.n_slots; j++) issue(j);
    fl_pdl_trigger();
    fl_pdl_wait();

    /* ── prologue: producer op + limb encoding of the input vector ── */
    Prolog P{a.in_mode, a.K, a.x, a.norm_w, a.pend, a.pend_w, 1.0f, 1.0f};
    float amax;
    if (a.in_mode == FL_IN_PLAIN) {
        amax = *a.absmax;
    } else {
        float ss = 0.0f, mx = 0.0f;
        if (a.in_mode == FL_IN_GEMMA_RESID) {
            float sp = 0.0f, dummy = 0.0f;
            for (int i = tid; i < a.K; i += FL_MV_THREADS) sp = fmaf(a.pend[i], a.pend[i], sp);
            fl_block_sum_max(sp, dummy, scratch);
            P.rms_p = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(sp, (float)a.K), 1e-6f));
        }
        for (int i = tid; i < a.K; i += FL_MV_THREADS) {
            float xi = a.in_mode == FL_IN_GEMMA_RESID ? P.resid(i) : a.x[i];
            if (a.in_mode == FL_IN_GEMMA_RESID && blockIdx.x == 0) a.resid_out[i] = xi;
            float wi = a.in_mode == FL_IN_RMSNORM ? a.norm_w[i] : __fadd_rn(a.norm_w[i], 1.0f);
            ss = fmaf(xi, xi, ss);
            mx = fmaxf(mx, fabsf(xi * wi));
        }
        fl_block_sum_max(ss, mx, scratch);
        P.rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)a.K), a.eps));
        amax = P.rms * mx * 1.00001f;
    }
    const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    if (tid == 0) s_scale = amax / 127.0f;
    for (int w = tid; w < n_chunks * 4; w += FL_MV_THREADS) {
        const int c = w >> 2, base = c * 32 + t * 8;
        float v[8];
        float hs = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            v[i] = base + i < a.K ? P.value(base + i) : 0.0f;
            hs += v[i];
        }
        encode_word(v, inv, xl + (size_t)c * FL_XENC_LIMB_BYTES, t);
        hs += __shfl_xor_sync(0xffffffffu, hs, 1);
        sxf[c * 4 + t] = (t & 1) ? 0.0f : hs;
    }
    __syncthreads();
    const float xscale = s_scale;

    /* ── main loop ── */
    float best_v = 0.0f;
    int best_i = 0x7fffffff;
    int j = 0;
    for (int it = 0; it < my_tiles; it++) {
        const int tile = (int)blockIdx.x + it * G;
        const int si = seg_of(a, tile);
        const FlMvSeg& sg = a.seg[si];
        float acc0 = 0.0f, acc1 = 0.0f, min0 = 0.0f, min1 = 0.0f;
        for (int kk = 0; kk < upt; kk++, j++) {
            const int slot = j % a.n_slots;
            if (!s_abort && !fl_mbar_wait(&wbar[slot], (uint32_t)((j / a.n_slots) & 1), a.err)) s_abort = 1;
            const uint8_t* u = wring + (size_t)slot * a.slot_bytes;
            process_any(sg.fmt, u, sg.expanded, warp + 8 * kk, xl, sxf, wstab, lane, acc0, acc1, min0, min1);
            __syncwarp();
            if (lane == 0 && j + a.n_slots < total) {
                fl_fence_proxy_async();
                issue(j + a.n_slots);
            }
        }
        const float wp = (t & 1) ? (1.0f / 2097152.0f) : (1.0f / 128.0f);
        float v0 = fmaf(acc0, wp * xscale, -min0), v1 = fmaf(acc1, wp * xscale, -min1);
        v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
        v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
        if (t == 0) {
            red[((it & 1) * FL_MV_WARPS + warp) * 16 + (lane >> 2)] = v0;
            red[((it & 1) * FL_MV_WARPS + warp) * 16 + (lane >> 2) + 8] = v1;
        }
        __syncthreads();
        if (warp == 0) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < FL_MV_WARPS; w++) v += red[((it & 1) * FL_MV_WARPS + w) * 16 + (lane & 15)];
            epilogue<EPI>(a, sg, si, tile, lane, v, best_v, best_i);
        }
    }

    if constexpr (EPI == FL_EPI_LOGITS) {
        __shared__ int s_last;
        if (tid == 0) {
            a.cta_best[blockIdx.x * 2] = best_v;
            a.cta_best[blockIdx.x * 2 + 1] = __int_as_float(best_i);
            __threadfence();
            s_last = atomicAdd(a.counter, 1) == G - 1;
        }
        __syncthreads();
        if (s_last && warp == 0) {
            __threadfence();
            float bv = 0.0f;
            int bi = 0x7fffffff;
            for (int b = lane; b < G; b += 32) {
                float v = __ldcg(&a.cta_best[b * 2]);
                int i = __float_as_int(__ldcg(&a.cta_best[b * 2 + 1]));
                if (i != 0x7fffffff && (bi == 0x7fffffff || fl_argmax_better(v, i, bv, bi))) {
                    bv = v;
                    bi = i;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (oi != 0x7fffffff && (bi == 0x7fffffff || fl_argmax_better(ov, oi, bv, bi))) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (lane == 0) {
                *a.argmax_out = bi;
                *a.counter = 0;
            }
        }
    }
}

template <int EPI>
cudaError_t configure_epi()
{
    /* the dynamic shared memory opt-in is per device */
    static unsigned long long done = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && ((done >> dev) & 1ull)) return cudaSuccess;
    e = cudaFuncSetAttribute(fl_mv_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e == cudaSuccess && dev < 64) done |= 1ull << dev;
    return e;
}

template <int EPI>
cudaError_t launch_epi(const FlMvArgs& a, int grid, size_t smem, cudaStream_t st, bool pdl)
{
    cudaError_t e = configure_epi<EPI>();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(FL_MV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fl_mv_kernel<EPI>, a);
}

} // namespace

size_t fl_mv_smem_bytes(const FlMvArgs& a)
{
    size_t n_chunks = (size_t)a.n_kb * 8;
    size_t off = (n_chunks * (FL_XENC_LIMB_BYTES + FL_XENC_SX_BYTES) + 127) & ~(size_t)127;
    off += (size_t)FL_MV_WARPS * a.n_slots * a.slot_bytes;
    off += (size_t)FL_MV_WARPS * a.n_slots * 8;
    off = (off + 15) & ~(size_t)15;
    off += (size_t)FL_MV_WARPS * 16 * kStabStride * 8;
    off += 2 * FL_MV_WARPS * 16 * 4;
    off += 64 * 4;
    return off;
}

cudaError_t fl_mv_configure()
{
    cudaError_t e = configure_epi<FL_EPI_STORE>();
    if (e == cudaSuccess) e = configure_epi<FL_EPI_RESID>();
    if (e == cudaSuccess) e = configure_epi<FL_EPI_QKV>();
    if (e == cudaSuccess) e = configure_epi<FL_EPI_GLU>();
    if (e == cudaSuccess) e = configure_epi<FL_EPI_LOGITS>();
    return e;
}

cudaError_t fl_launch_matvec(const FlMvArgs& a, int grid, cudaStream_t st, bool pdl)
{
    size_t smem = fl_mv_smem_bytes(a);
    switch (a.epi) {
    case FL_EPI_STORE: return launch_epi<FL_EPI_STORE>(a, grid, smem, st, pdl);
    case FL_EPI_RESID: return launch_epi<FL_EPI_RESID>(a, grid, smem, st, pdl);
    case FL_EPI_QKV: return launch_epi<FL_EPI_QKV>(a, grid, smem, st, pdl);
    case FL_EPI_GLU: return launch_epi<FL_EPI_GLU>(a, grid, smem, st, pdl);
    default: return launch_epi<FL_EPI_LOGITS>(a, grid, smem, st, pdl);
    }
}
