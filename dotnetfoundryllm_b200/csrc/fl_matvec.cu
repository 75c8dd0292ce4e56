/*
 * fl_matvec.cu — one dequant-matvec as its own launch (fl_matvec, and the
 * building block the token step's phases share through fl_mv_core.cuh).
 *
 * Replaces LinearProjection over dequantized F32 weights
 * (src/DotNetFoundryLLM.Architectures/LlamaForwardPass.cs:237-260).
 *
 *  - grid = min(#tiles, #SMs), 8 warps per CTA.  CTA b owns tiles b, b+G, ...;
 *    warp w owns k-blocks w, w+8, ... of each of them.
 *  - every warp streams its own units (16 rows x 256 columns) HBM → shared
 *    memory with 1-D bulk async copies into a private ring of mbarrier slots.
 *  - each warp encodes the input values of its own k-blocks into 3 int8 limbs
 *    and runs one m16n8k32 int8 MMA per (16 rows x 32 values) chunk; the
 *    integer sums are scaled by the format's (d, sc, m) per unit.
 *  - the partial sums of a tile's warps are combined by the last warp to
 *    finish it, which also runs the consumer op.
 */
#include "fl_mv_core.cuh"

using namespace flcore;

namespace {

/* Shared-memory carve-up, identical on host and device. */
struct Layout {
    size_t xl, xs, xsum, zero, ring, bars, red, cnt, done, best, scratch, total;
};

__host__ __device__ inline Layout smem_layout(int n_kb, int n_slots, int slot_bytes)
{
    Layout L;
    const size_t nc = (size_t)n_kb * 8;
    L.xl = 0;                                   /* [chunk][limb 0..2][t][8 B] */
    L.xs = L.xl + nc * FL_XENC_LIMB_BYTES;      /* [chunk][t] short2 limb sums of the lane's half */
    L.xsum = L.xs + nc * FL_XENC_LSUM_BYTES;    /* [chunk][half] float sums */
    L.zero = L.xsum + nc * FL_XENC_HSUM_BYTES;  /* zero B fragments */
    L.ring = (L.zero + FL_XENC_ZERO_BYTES + 127) & ~(size_t)127;
    L.bars = L.ring + (size_t)FL_MV_WARPS * n_slots * slot_bytes;
    L.red = L.bars + (size_t)FL_MV_WARPS * n_slots * 8;
    L.cnt = L.red + (size_t)kRedSlots * FL_MV_WARPS * 16 * 4;
    L.done = L.cnt + kRedSlots * 4;
    L.best = L.done + kRedSlots * 4;
    L.scratch = L.best + FL_MV_WARPS * 8;
    L.total = L.scratch + 64 * 4;
    return L;
}

template <int EPI>
__global__ void __launch_bounds__(FL_MV_THREADS, 1) fl_mv_kernel(const __grid_constant__ FlMvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red2[64];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const Layout Ls = smem_layout(a.n_kb, a.n_slots, a.slot_bytes);
    uint8_t* xl = smem + Ls.xl;
    short2* xs = reinterpret_cast<short2*>(smem + Ls.xs);
    float* xsum = reinterpret_cast<float*>(smem + Ls.xsum);
    uint8_t* zero = smem + Ls.zero;
    uint8_t* ring = smem + Ls.ring;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Ls.bars);
    float* red = reinterpret_cast<float*>(smem + Ls.red);
    int* cnt = reinterpret_cast<int*>(smem + Ls.cnt);
    int* done = reinterpret_cast<int*>(smem + Ls.done);
    float* best = reinterpret_cast<float*>(smem + Ls.best);

    const int G = gridDim.x;
    const int my_tiles = a.n_tiles > (int)blockIdx.x ? (a.n_tiles - (int)blockIdx.x + G - 1) / G : 0;
    const int upt = warp < a.n_kb ? (a.n_kb - warp + FL_MV_WARPS - 1) / FL_MV_WARPS : 0;
    const int total = my_tiles * upt;
    uint8_t* wring = ring + (size_t)warp * a.n_slots * a.slot_bytes;
    uint64_t* wbar = bars + warp * a.n_slots;

    if (lane == 0)
        for (int i = 0; i < a.n_slots; i++) fl_mbar_init(&wbar[i], 1);
    if (tid < kRedSlots) {
        cnt[tid] = 0;
        done[tid] = 0;
    }
    for (int i = tid; i < FL_XENC_ZERO_BYTES; i += FL_MV_THREADS) zero[i] = 0;
    fl_fence_mbar_init();
    __syncthreads();

    auto issue = [&](int j) {
        const int tile = (int)blockIdx.x + (j / upt) * G;
        const int kb = warp + FL_MV_WARPS * (j % upt);
        const FlMvSeg& sg = a.seg[seg_of(a, tile)];
        const uint8_t* src = sg.w + ((size_t)(tile - sg.tile0) * a.n_kb + kb) * sg.unit_bytes;
        const int slot = j % a.n_slots;
        fl_mbar_expect_tx(&wbar[slot], (uint32_t)sg.unit_bytes);
        fl_bulk_g2s(wring + (size_t)slot * a.slot_bytes, src, (uint32_t)sg.unit_bytes, &wbar[slot]);
    };

    if (lane == 0)
        for (int j = 0; j < total && j < a.n_slots; j++) issue(j);
    fl_pdl_trigger();
    fl_pdl_wait();

    Prolog P{a.in_mode, a.K, a.x, a.norm_w, a.pend, a.pend_w, 1.0f, 1.0f};
    float amax;
    if (a.in_mode == FL_IN_PLAIN) {
        amax = __ldcg(a.absmax);
    } else {
        float ss = 0.0f, mx = 0.0f;
        if (a.in_mode == FL_IN_GEMMA_RESID) {
            float sp = 0.0f, dummy = 0.0f;
            for (int i = tid; i < a.K; i += FL_MV_THREADS) sp = fmaf(__ldcg(a.pend + i), __ldcg(a.pend + i), sp);
            fl_block_sum_max(sp, dummy, s_red2);
            P.rms_p = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(sp, (float)a.K), 1e-6f));
        }
        for (int i = tid; i < a.K; i += FL_MV_THREADS) {
            float xi = a.in_mode == FL_IN_GEMMA_RESID ? P.resid(i) : __ldcg(a.x + i);
            if (a.in_mode == FL_IN_GEMMA_RESID && blockIdx.x == 0) a.resid_out[i] = xi;
            float wi = a.in_mode == FL_IN_RMSNORM ? a.norm_w[i] : __fadd_rn(a.norm_w[i], 1.0f);
            ss = fmaf(xi, xi, ss);
            mx = fmaxf(mx, fabsf(xi * wi));
        }
        fl_block_sum_max(ss, mx, s_red2);
        P.rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)a.K), a.eps));
        amax = P.rms * mx * 1.00001f;
    }
    const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    const float xscale = amax / 127.0f;
    for (int kk = 0; kk < upt; kk++) encode_kblock(P, warp + FL_MV_WARPS * kk, inv, lane, xl, xs, xsum);
    __syncwarp();
    const int pos = (EPI == FL_EPI_QKV) ? __ldcg(a.pos) : 0;

    const int limb = g & 3;
    const bool bval = (limb < 3) && ((g >> 2) == (t >> 1));
    const uint8_t* bptr = xl + (limb * 4 + t) * 8;
    const float wlane = ((t & 1) ? (1.0f / 16384.0f) : 1.0f) * xscale;

    float best_v = 0.0f;
    int best_i = 0x7fffffff;
    int j = 0;
    for (int it = 0; it < my_tiles; it++) {
        const int tile = (int)blockIdx.x + it * G;
        const int si = seg_of(a, tile);
        const FlMvSeg& sg = a.seg[si];
        Acc A{0.0f, 0.0f, 0.0f, 0.0f};
        for (int kk = 0; kk < upt; kk++, j++) {
            const int slot = j % a.n_slots;
            fl_mbar_wait(&wbar[slot], (uint32_t)((j / a.n_slots) & 1), a.err);
            const uint8_t* u = wring + (size_t)slot * a.slot_bytes;
            process_any(sg.fmt, sg.expanded, u, warp + FL_MV_WARPS * kk,
                        unit_bptr(bptr, bval, zero, warp + FL_MV_WARPS * kk), xs, xsum, lane, A);
            __syncwarp();
            if (lane == 0 && j + a.n_slots < total) {
                fl_fence_proxy_async();
                issue(j + a.n_slots);
            }
        }
        float v0 = fmaf(A.res0, wlane, -A.m0), v1 = fmaf(A.res1, wlane, -A.m1);
        v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
        v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
        const int slot = it % kRedSlots, gen = it / kRedSlots;
        if (lane == 0) wait_slot(&done[slot], gen, a.err);
        __syncwarp();
        float* rs = red + (size_t)slot * FL_MV_WARPS * 16 + warp * 16;
        if (t == 0) {
            rs[g] = v0;
            rs[g + 8] = v1;
        }
        __threadfence_block();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&cnt[slot], 1) == FL_MV_WARPS - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            const volatile float* rv = red + (size_t)slot * FL_MV_WARPS * 16;
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < FL_MV_WARPS; w++) v += rv[w * 16 + (lane & 15)];
            __syncwarp();
            if (lane == 0) {
                cnt[slot] = 0;
                __threadfence_block();
                atomicAdd(&done[slot], 1);
            }
            epilogue<EPI>(a, sg, si, tile, lane, v, pos, best_v, best_i);
        }
    }

    if constexpr (EPI == FL_EPI_LOGITS) {
        __shared__ int s_last;
        if (lane == 0) {
            best[warp * 2] = best_v;
            best[warp * 2 + 1] = __int_as_float(best_i);
        }
        __syncthreads();
        if (tid == 0) {
            float bv = 0.0f;
            int bi = 0x7fffffff;
            for (int w = 0; w < FL_MV_WARPS; w++) {
                float v = best[w * 2];
                int i = __float_as_int(best[w * 2 + 1]);
                if (i != 0x7fffffff && (bi == 0x7fffffff || fl_argmax_better(v, i, bv, bi))) {
                    bv = v;
                    bi = i;
                }
            }
            a.cta_best[blockIdx.x * 2] = bv;
            a.cta_best[blockIdx.x * 2 + 1] = __int_as_float(bi);
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
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, fl_mv_kernel<EPI>);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fl_mv_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)fa.sharedSizeBytes);
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

size_t fl_mv_smem_bytes(const FlMvArgs& a) { return smem_layout(a.n_kb, a.n_slots, a.slot_bytes).total; }

size_t fl_mv_fixed_smem_bytes(int n_kb) { return smem_layout(n_kb, 0, 0).total; }

cudaError_t fl_mv_configure()
{
    cudaError_t e = configure_epi<FL_EPI_STORE>();
    if (e == cudaSuccess) e = configure_epi<FL_EPI_RESID>();
    if (e == cudaSuccess) e = configure_epi<FL_EPI_QKV>();
    if (e == cudaSuccess) e = configure_epi<FL_EPI_GLU>();
    if (e == cudaSuccess) e = configure_epi<FL_EPI_LOGITS>();
    return e;
}

void fl_mv_ring_config(FlMvArgs& a)
{
    int maxu = 0;
    for (int i = 0; i < a.n_seg; i++) maxu = a.seg[i].unit_bytes > maxu ? a.seg[i].unit_bytes : maxu;
    a.slot_bytes = (maxu + 127) & ~127;
    const long budget = 112 * 1024 - (long)fl_mv_fixed_smem_bytes(a.n_kb);
    const long n = budget / ((long)FL_MV_WARPS * a.slot_bytes);
    a.n_slots = (int)(n < 2 ? 2 : (n > 8 ? 8 : n));
}

cudaError_t fl_launch_matvec(const FlMvArgs& a, int grid, cudaStream_t st, bool pdl)
{
    /* every unit must fit a ring slot */
    if (a.n_slots < 1 || a.n_seg < 1 || a.n_seg > FL_MV_MAX_SEG) return cudaErrorInvalidValue;
    for (int i = 0; i < a.n_seg; i++)
        if (a.seg[i].unit_bytes <= 0 || a.seg[i].unit_bytes > a.slot_bytes || (a.seg[i].unit_bytes & 15))
            return cudaErrorInvalidValue;
    size_t smem = fl_mv_smem_bytes(a);
    switch (a.epi) {
    case FL_EPI_STORE: return launch_epi<FL_EPI_STORE>(a, grid, smem, st, pdl);
    case FL_EPI_RESID: return launch_epi<FL_EPI_RESID>(a, grid, smem, st, pdl);
    case FL_EPI_QKV: return launch_epi<FL_EPI_QKV>(a, grid, smem, st, pdl);
    case FL_EPI_GLU: return launch_epi<FL_EPI_GLU>(a, grid, smem, st, pdl);
    default: return launch_epi<FL_EPI_LOGITS>(a, grid, smem, st, pdl);
    }
}
