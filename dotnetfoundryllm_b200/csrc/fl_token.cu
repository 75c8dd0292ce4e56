/*
 * fl_token.cu — one decode step (IForwardPass.Forward + greedy ArgMax) as one
 * persistent cooperative kernel.
 *
 * The step is a list of phases (embedding row, then per layer: QKV matvec,
 * attention, output projection, gate/up, down; then the LM head), the same
 * ops as LlamaForwardPass.Forward (src/DotNetFoundryLLM.Architectures/
 * LlamaForwardPass.cs:82-130) and its Mistral/Gemma2/Qwen2 copies.  One CTA
 * per SM runs all of them:
 *
 *  - a producer warp walks every matvec phase's weight units in the order the
 *    consumers will need them and streams them HBM → shared memory with 1-D
 *    bulk async copies into one ring of mbarrier slots.  It never waits for a
 *    phase boundary, so the weights of the next projection are already in
 *    shared memory while the current one drains and the grid synchronizes;
 *  - 15 consumer warps take the units round-robin, run the int8 tensor-core
 *    dequant-matvec (fl_mv_core.cuh), reduce each 16-row tile across warps and
 *    apply its epilogue;
 *  - phases are separated by a grid barrier (arrival counter in global memory,
 *    bounded spin); data produced by an earlier phase is read through L2.
 *
 * All CTAs must be resident at once: the kernel is launched cooperatively with
 * one CTA per SM.  Every wait is bounded and records FL_DEV_ERR_TIMEOUT instead
 * of hanging.
 */
#include "fl_mv_core.cuh"

using namespace flcore;

namespace {

constexpr int NW = FL_TK_WARPS;          /* consumer warps */
constexpr int NT = (NW + 1) * 32;        /* + producer warp */
constexpr int RED = 8;                   /* tile reductions in flight */

struct TkLayout {
    size_t ring, full, empty, scratch, zero, red, cnt, done, best, misc, total;
};

__host__ __device__ inline TkLayout tk_layout(int n_slots, int slot_bytes, size_t scratch_bytes)
{
    TkLayout L;
    L.ring = 0;
    L.full = L.ring + (size_t)n_slots * slot_bytes;
    L.empty = L.full + (size_t)n_slots * 8;
    L.scratch = (L.empty + (size_t)n_slots * 8 + 127) & ~(size_t)127;
    L.zero = L.scratch + ((scratch_bytes + 15) & ~(size_t)15);
    L.red = L.zero + 16;
    L.cnt = L.red + (size_t)RED * NW * 16 * 4;
    L.done = L.cnt + RED * 4;
    L.best = L.done + RED * 4;
    L.misc = L.best + NW * 8;
    L.total = L.misc + 64 * 4;
    return L;
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"r"(NW * 32) : "memory"); }

__device__ __forceinline__ int ld_acquire(const int* p)
{
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(fl_smem_u32(bar)) : "memory");
}

/* All CTAs finish phase k before any starts phase k+1.  Bounded: gives up after
 * ~2 s, records a timeout and lets the kernel run to its end. */
__device__ void grid_sync(int* bar, int target, int* err)
{
    consumer_sync();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(bar, 1);
        if (ld_acquire(bar) < target) {
            const uint64_t t0 = fl_globaltimer();
            for (uint32_t it = 0;; it++) {
                if (ld_acquire(bar) >= target) break;
                __nanosleep(64);
                if ((it & 63u) == 0 && (fl_globaltimer() - t0 > 2000000000ull || it > (1u << 26))) {
                    atomicExch(err, FL_DEV_ERR_TIMEOUT);
                    break;
                }
            }
        }
        __threadfence();
    }
    consumer_sync();
}

/* Block reduction over the consumer threads (sum, max). */
__device__ __forceinline__ void consumer_sum_max(float& s, float& m, float* scratch)
{
    s = fl_warp_sum(s);
    m = fl_warp_max(m);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    consumer_sync();
    if (lane == 0) {
        scratch[warp] = s;
        scratch[32 + warp] = m;
    }
    consumer_sync();
    float ts = 0.0f, tm = 0.0f;
    for (int w = 0; w < NW; w++) {
        ts += scratch[w];
        tm = fmaxf(tm, scratch[32 + w]);
    }
    s = ts;
    m = tm;
}

/* ── phases ─────────────────────────────────────────────────────────────── */

__device__ void phase_embed(const FlEmbedArgs& e, int* err)
{
    /* TokenEmbedding.AsSpan(tokenId * h, h).CopyTo(_x) (LlamaForwardPass.cs:96) */
    int tok = __ldcg(e.token);
    if (tok < 0 || tok >= e.vocab) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, FL_DEV_ERR_TOKEN);
        tok = 0;
    }
    const int stride = gridDim.x * NW * 32;
    for (int i = blockIdx.x * NW * 32 + threadIdx.x; i < e.hidden; i += stride)
        e.x[i] = fl_dequant_elem(e.ggml_type, e.raw, (int64_t)tok * e.hidden + i);
    for (int i = blockIdx.x * NW * 32 + threadIdx.x; i < e.zero_n; i += stride) e.zero_buf[i] = 0.0f;
}

/* Attention for items (kv head, split) b, b+G, ...: the consumer warps split the
 * item's keys; per-warp online softmax; merged in shared memory; the last item
 * of a kv head merges the splits (ComputeAttention, LlamaForwardPass.cs:158-211;
 * MistralForwardPass.cs:186-240; Gemma2ForwardPass.cs:126-185). */
template <int HD, int GRP>
__device__ void phase_attn_t(const FlAttnArgs& a, float* scr, int* err)
{
    constexpr int PER = HD / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv_dim = a.n_kv * HD;
    float* sq = scr;                                   /* [GRP*HD] */
    float* sml = sq + GRP * HD;                        /* [NW][GRP][2] */
    float* sacc = sml + NW * GRP * 2;                  /* [NW][GRP][HD] */
    __shared__ int s_last;
    const int seq = __ldcg(a.pos) + 1;
    int start = 0;
    if (a.window < seq) start = seq - a.window;
    const int L = seq - start;
    const int per = (L + a.n_split - 1) / a.n_split;
    const float inv_cap = a.softcap > 0.0f ? 1.0f / a.softcap : 0.0f;
    const int n_items = a.n_kv * a.n_split;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int kvh = item / a.n_split, split = item % a.n_split;
        const int k0 = start + split * per, k1 = min(seq, k0 + per);
        for (int i = threadIdx.x; i < GRP * HD; i += NW * 32) sq[i] = __ldcg(a.q + (size_t)kvh * GRP * HD + i);
        consumer_sync();
        float m[GRP], l[GRP], acc[GRP][PER];
#pragma unroll
        for (int h = 0; h < GRP; h++) {
            m[h] = -INFINITY;
            l[h] = 0.0f;
#pragma unroll
            for (int p = 0; p < PER; p++) acc[h][p] = 0.0f;
        }
        for (int t = k0 + warp; t < k1; t += NW) {
            const float* kr = a.k_cache + (size_t)t * kv_dim + (size_t)kvh * HD;
            const float* vr = a.v_cache + (size_t)t * kv_dim + (size_t)kvh * HD;
            float kk[PER], vv[PER];
#pragma unroll
            for (int p = 0; p < PER; p++) {
                kk[p] = __ldcg(kr + lane + 32 * p);
                vv[p] = __ldcg(vr + lane + 32 * p);
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
#pragma unroll
        for (int h = 0; h < GRP; h++) {
            if (lane == 0) {
                sml[(warp * GRP + h) * 2] = m[h];
                sml[(warp * GRP + h) * 2 + 1] = l[h];
            }
#pragma unroll
            for (int p = 0; p < PER; p++) sacc[(warp * GRP + h) * HD + lane + 32 * p] = acc[h][p];
        }
        consumer_sync();
        float* part = a.part + (size_t)item * GRP * (HD + 2);
        for (int i = threadIdx.x; i < GRP * HD; i += NW * 32) {
            const int h = i / HD, d = i % HD;
            float M = -INFINITY;
            for (int w = 0; w < NW; w++) M = fmaxf(M, sml[(w * GRP + h) * 2]);
            float Ls = 0.0f, O = 0.0f;
            for (int w = 0; w < NW; w++) {
                const float mw = sml[(w * GRP + h) * 2];
                const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
                Ls = fmaf(sml[(w * GRP + h) * 2 + 1], f, Ls);
                O = fmaf(sacc[(w * GRP + h) * HD + d], f, O);
            }
            part[h * (HD + 2) + 2 + d] = O;
            if (d == 0) {
                part[h * (HD + 2)] = M;
                part[h * (HD + 2) + 1] = Ls;
            }
        }
        __threadfence();
        consumer_sync();
        if (threadIdx.x == 0) s_last = atomicAdd(&a.counter[kvh], 1) == a.n_split - 1;
        consumer_sync();
        if (s_last) {
            __threadfence();
            float amax = 0.0f;
            const float* pk = a.part + (size_t)kvh * a.n_split * GRP * (HD + 2);
            for (int i = threadIdx.x; i < GRP * HD; i += NW * 32) {
                const int h = i / HD, d = i % HD;
                float M = -INFINITY;
                for (int s = 0; s < a.n_split; s++) M = fmaxf(M, __ldcg(&pk[((size_t)s * GRP + h) * (HD + 2)]));
                float Ls = 0.0f, O = 0.0f;
                for (int s = 0; s < a.n_split; s++) {
                    const float* ps = pk + ((size_t)s * GRP + h) * (HD + 2);
                    const float ms = __ldcg(&ps[0]);
                    const float f = ms == -INFINITY ? 0.0f : expf(ms - M);
                    Ls = fmaf(__ldcg(&ps[1]), f, Ls);
                    O = fmaf(__ldcg(&ps[2 + d]), f, O);
                }
                const float o = Ls > 0.0f ? O / Ls : 0.0f;
                a.out[((size_t)kvh * GRP + h) * HD + d] = o;
                amax = fmaxf(amax, fabsf(o));
            }
            amax = fl_warp_max(amax);
            if (lane == 0) atomicMax(reinterpret_cast<int*>(a.out_absmax), __float_as_int(amax));
            if (threadIdx.x == 0) a.counter[kvh] = 0;
        }
        consumer_sync();
    }
}

template <int HD>
__device__ void phase_attn_hd(const FlAttnArgs& a, float* scr, int* err)
{
    /* group sizes of the supported configurations (head_dim 256 stops at 4) */
    switch (a.n_heads / a.n_kv) {
    case 1: phase_attn_t<HD, 1>(a, scr, err); break;
    case 2: phase_attn_t<HD, 2>(a, scr, err); break;
    case 4: phase_attn_t<HD, 4>(a, scr, err); break;
    default:
        if constexpr (HD <= 128) phase_attn_t<HD, 8>(a, scr, err);
        break;
    }
}

__device__ void phase_attn(const FlAttnArgs& a, float* scr, int* err)
{
    switch (a.head_dim) {
    case 64: phase_attn_hd<64>(a, scr, err); break;
    case 128: phase_attn_hd<128>(a, scr, err); break;
    default: phase_attn_hd<256>(a, scr, err); break;
    }
}

struct Ring {
    uint8_t* base;
    uint64_t* full;
    uint64_t* empty;
    int n_slots, slot_bytes;
};

/* Producer: the CTA's weight units of every matvec phase, in consumption order. */
__device__ void producer(const FlTokenArgs& ta, const Ring& R)
{
    if ((threadIdx.x & 31) != 0) return;
    const int G = gridDim.x;
    uint32_t u = 0;
    for (int p = 0; p < ta.n_phases; p++) {
        const FlPhase& ph = ta.phases[p];
        if (ph.kind != FL_PH_MATVEC) continue;
        const FlMvArgs& a = ph.mv;
        const int my_tiles = a.n_tiles > (int)blockIdx.x ? (a.n_tiles - (int)blockIdx.x + G - 1) / G : 0;
        for (int it = 0; it < my_tiles; it++) {
            const int tile = (int)blockIdx.x + it * G;
            const FlMvSeg& sg = a.seg[seg_of(a, tile)];
            const uint8_t* src = sg.w + (size_t)(tile - sg.tile0) * a.n_kb * sg.unit_bytes;
            for (int kb = 0; kb < a.n_kb; kb++, u++) {
                const int slot = (int)(u % (uint32_t)R.n_slots);
                if (u >= (uint32_t)R.n_slots)
                    fl_mbar_wait(&R.empty[slot], ((u / R.n_slots) - 1) & 1, ta.err);
                fl_mbar_expect_tx(&R.full[slot], (uint32_t)sg.unit_bytes);
                fl_bulk_g2s(R.base + (size_t)slot * R.slot_bytes, src + (size_t)kb * sg.unit_bytes,
                            (uint32_t)sg.unit_bytes, &R.full[slot]);
            }
        }
    }
}

} // namespace

__global__ void __launch_bounds__(NT, 1) fl_token_kernel(const __grid_constant__ FlTokenArgs ta)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const TkLayout Ls = tk_layout(ta.n_slots, ta.slot_bytes, ta.scratch_bytes);
    Ring R{smem + Ls.ring, reinterpret_cast<uint64_t*>(smem + Ls.full), reinterpret_cast<uint64_t*>(smem + Ls.empty),
           ta.n_slots, ta.slot_bytes};
    uint8_t* scratch = smem + Ls.scratch;
    uint8_t* zero = smem + Ls.zero;
    float* red = reinterpret_cast<float*>(smem + Ls.red);
    int* cnt = reinterpret_cast<int*>(smem + Ls.cnt);
    int* done = reinterpret_cast<int*>(smem + Ls.done);
    float* best = reinterpret_cast<float*>(smem + Ls.best);
    float* misc = reinterpret_cast<float*>(smem + Ls.misc);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int G = gridDim.x;

    if (tid == 0) {
        for (int i = 0; i < ta.n_slots; i++) {
            fl_mbar_init(&R.full[i], 1);
            fl_mbar_init(&R.empty[i], 1);
        }
    }
    for (int i = tid; i < RED * NW * 16; i += NT) red[i] = 0.0f;
    if (tid < RED) {
        cnt[tid] = 0;
        done[tid] = 0;
    }
    if (tid < 16) zero[tid] = 0;
    fl_fence_mbar_init();
    __syncthreads();

    if (warp == NW) {
        producer(ta, R);
        return;
    }

    uint32_t U = 0; /* unit counter (same sequence as the producer) */
    int T = 0;      /* tile counter across phases (reduction slots) */
    float best_v = 0.0f;
    int best_i = 0x7fffffff;
    for (int p = 0; p < ta.n_phases; p++) {
        const FlPhase& ph = ta.phases[p];
        if (p > 0) grid_sync(ta.bar, p * G, ta.err);
        if (ta.timestamps && blockIdx.x == 0 && tid == 0) ta.timestamps[p] = fl_globaltimer();
        if (ph.kind == FL_PH_EMBED) {
            phase_embed(ph.em, ta.err);
            continue;
        }
        if (ph.kind == FL_PH_ATTN) {
            phase_attn(ph.at, reinterpret_cast<float*>(scratch), ta.err);
            continue;
        }
        /* ── matvec phase ── */
        const FlMvArgs& a = ph.mv;
        uint8_t* xl = scratch;
        const size_t nc = (size_t)a.n_kb * 8;
        int2* xs = reinterpret_cast<int2*>(scratch + nc * FL_XENC_LIMB_BYTES);
        float* xsum = reinterpret_cast<float*>(scratch + nc * (FL_XENC_LIMB_BYTES + 32));
        Prolog P{a.in_mode, a.K, a.x, a.norm_w, a.pend, a.pend_w, 1.0f, 1.0f};
        float amax;
        if (a.in_mode == FL_IN_PLAIN) {
            amax = __ldcg(a.absmax);
        } else {
            float ss = 0.0f, mx = 0.0f;
            if (a.in_mode == FL_IN_GEMMA_RESID) {
                float sp = 0.0f, dummy = 0.0f;
                for (int i = tid; i < a.K; i += NW * 32) {
                    const float v = __ldcg(a.pend + i);
                    sp = fmaf(v, v, sp);
                }
                consumer_sum_max(sp, dummy, misc);
                P.rms_p = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(sp, (float)a.K), 1e-6f));
            }
            for (int i = tid; i < a.K; i += NW * 32) {
                const float xi = a.in_mode == FL_IN_GEMMA_RESID ? P.resid(i) : __ldcg(a.x + i);
                if (a.in_mode == FL_IN_GEMMA_RESID && blockIdx.x == 0) a.resid_out[i] = xi;
                const float wi = a.in_mode == FL_IN_RMSNORM ? a.norm_w[i] : __fadd_rn(a.norm_w[i], 1.0f);
                ss = fmaf(xi, xi, ss);
                mx = fmaxf(mx, fabsf(xi * wi));
            }
            consumer_sum_max(ss, mx, misc);
            P.rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)a.K), a.eps));
            amax = P.rms * mx * 1.00001f;
        }
        const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
        const float xscale = amax / 127.0f;
        for (int kb = warp; kb < a.n_kb; kb += NW) encode_kblock(P, kb, inv, lane, xl, xs, xsum);
        consumer_sync();
        const int pos = a.epi == FL_EPI_QKV ? __ldcg(a.pos) : 0;
        const int limb = g & 3;
        const bool bval = (limb < 3) && ((g >> 2) == (t >> 1));
        const uint8_t* bptr = bval ? xl + (limb * 4 + t) * 8 : zero;
        const int bstride = bval ? FL_XENC_LIMB_BYTES : 0;
        const float wlane = ((t & 1) ? (1.0f / 16384.0f) : 1.0f) * xscale;
        const int my_tiles = a.n_tiles > (int)blockIdx.x ? (a.n_tiles - (int)blockIdx.x + G - 1) / G : 0;

        for (int it = 0; it < my_tiles; it++, T++) {
            const int tile = (int)blockIdx.x + it * G;
            const int si = seg_of(a, tile);
            const FlMvSeg& sg = a.seg[si];
            Acc A{0.0f, 0.0f, 0.0f, 0.0f};
            int cw = 0;
            /* units U .. U+n_kb-1; this warp takes those with u % NW == warp */
            int kb = (int)((warp - (int)(U % NW) + NW) % NW);
            for (; kb < a.n_kb; kb += NW) {
                const uint32_t u = U + kb;
                const int slot = (int)(u % (uint32_t)R.n_slots);
                fl_mbar_wait(&R.full[slot], (u / R.n_slots) & 1, ta.err);
                process_any(sg.fmt, sg.expanded, R.base + (size_t)slot * R.slot_bytes, kb, bptr, bstride, xs, xsum,
                            lane, A);
                __syncwarp();
                if (lane == 0) mbar_arrive(&R.empty[slot]);
                cw++;
            }
            U += a.n_kb;
            if (cw == 0) continue;
            float v0 = fmaf(A.res0, wlane, -A.m0), v1 = fmaf(A.res1, wlane, -A.m1);
            v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
            v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
            v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
            v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
            const int slot = T % RED, gen = T / RED;
            if (lane == 0) wait_slot(&done[slot], gen, ta.err);
            __syncwarp();
            float* rs = red + (size_t)slot * NW * 16 + warp * 16;
            if (t == 0) {
                rs[g] = v0;
                rs[g + 8] = v1;
            }
            __threadfence_block();
            __syncwarp();
            int last = 0;
            if (lane == 0) last = atomicAdd(&cnt[slot], cw) + cw == a.n_kb;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence_block();
                volatile float* rv = red + (size_t)slot * NW * 16;
                float v = 0.0f;
#pragma unroll
                for (int w = 0; w < NW; w++) v += rv[w * 16 + (lane & 15)];
                __syncwarp();
                for (int i = lane; i < NW * 16; i += 32) rv[i] = 0.0f;
                __syncwarp();
                if (lane == 0) {
                    cnt[slot] = 0;
                    __threadfence_block();
                    atomicAdd(&done[slot], 1);
                }
                epilogue_any(a, sg, si, tile, lane, v, pos, best_v, best_i);
            }
        }
        if (a.epi == FL_EPI_LOGITS) {
            /* greedy ArgMax (TensorPrimitives.IndexOfMax): per CTA, then across CTAs */
            __shared__ int s_last;
            if (lane == 0) {
                best[warp * 2] = best_v;
                best[warp * 2 + 1] = __int_as_float(best_i);
            }
            consumer_sync();
            if (tid == 0) {
                float bv = 0.0f;
                int bi = 0x7fffffff;
                for (int w = 0; w < NW; w++) {
                    const float v = best[w * 2];
                    const int i = __float_as_int(best[w * 2 + 1]);
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
            consumer_sync();
            if (s_last && warp == 0) {
                __threadfence();
                float bv = 0.0f;
                int bi = 0x7fffffff;
                for (int b = lane; b < G; b += 32) {
                    const float v = __ldcg(&a.cta_best[b * 2]);
                    const int i = __float_as_int(__ldcg(&a.cta_best[b * 2 + 1]));
                    if (i != 0x7fffffff && (bi == 0x7fffffff || fl_argmax_better(v, i, bv, bi))) {
                        bv = v;
                        bi = i;
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (oi != 0x7fffffff && (bi == 0x7fffffff || fl_argmax_better(ov, oi, bv, bi))) {
                        bv = ov;
                        bi = oi;
                    }
                }
                if (lane == 0) {
                    *a.argmax_out = bi;
                    *a.counter = 0;
                    /* the device-resident decode loop: next token, next position */
                    if (ta.advance) {
                        const int s = __ldcg(ta.step);
                        if (ta.out_tokens) ta.out_tokens[s] = bi;
                        *ta.step = s + 1;
                        *ta.token = bi;
                        *ta.pos = __ldcg(ta.pos) + 1;
                    }
                    if (ta.timestamps) ta.timestamps[ta.n_phases] = fl_globaltimer();
                }
            }
        }
    }
}

size_t fl_token_smem_bytes(int n_slots, int slot_bytes, size_t scratch_bytes)
{
    return tk_layout(n_slots, slot_bytes, scratch_bytes).total;
}

cudaError_t fl_token_configure(int* max_dyn_smem)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, fl_token_kernel);
    if (e != cudaSuccess) return e;
    const int avail = optin - (int)fa.sharedSizeBytes;
    e = cudaFuncSetAttribute(fl_token_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, avail);
    if (e == cudaSuccess && max_dyn_smem) *max_dyn_smem = avail;
    return e;
}

cudaError_t fl_launch_token(const FlTokenArgs& ta, int grid, size_t smem, cudaStream_t st)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fl_token_kernel, ta);
}

const void* fl_token_kernel_ptr() { return reinterpret_cast<const void*>(fl_token_kernel); }
