/*
 * fl_token.cuh — one decode step (IForwardPass.Forward + greedy ArgMax) as one
 * persistent cooperative kernel.
 *
 * The step is a list of phases (embedding row, then per layer: QKV matvec,
 * attention, output projection, gate/up, down; then the LM head), the same
 * ops as LlamaForwardPass.Forward (src/DotNetFoundryLLM.Architectures/
 * LlamaForwardPass.cs:82-130) and its Mistral/Gemma2/Qwen2 copies.  One CTA
 * per SM runs all of them, 16 warps each:
 *
 *  - in a matvec phase the CTA's units (16 rows x 256 columns of weights) are
 *    split into 16 contiguous ranges, one per warp (stream-K inside the CTA).
 *    A tile inside one warp's range is finished by that warp alone; the at
 *    most two tiles a range shares with its neighbours are summed in warp
 *    order by whichever contributor finishes last, so every result is
 *    deterministic;
 *  - each warp streams its own units HBM → shared memory with 1-D bulk async
 *    copies into a private ring of mbarrier slots.  Its lane 0 refills a slot
 *    as soon as the unit in it has been copied to registers, running ahead
 *    through the warp's ranges of the following matvec phases, so the next
 *    projection's weights are in flight while the current phase drains and the
 *    grid synchronizes;
 *  - phases are separated by a grid barrier (arrival counter in global memory,
 *    bounded spin); data produced by an earlier phase is read through L2.
 *
 * All CTAs must be resident at once: the kernel is launched cooperatively with
 * one CTA per SM.  Every wait is bounded and records FL_DEV_ERR_TIMEOUT instead
 * of hanging.
 */
#ifndef FL_TOKEN_CUH
#define FL_TOKEN_CUH

#include "fl_mv_core.cuh"

namespace fltk {
namespace { /* internal linkage: the header is compiled into several units */

using namespace flcore;

constexpr int NW = FL_TK_WARPS;          /* warps */
constexpr int NC = NW * 32;              /* threads */
constexpr int NT = NC;
constexpr int TCNT = FL_TK_MAX_TILES;    /* per-CTA tiles of one phase */

/* Lane 0's cursor over its warp's units of every matvec phase, in the order the
 * warp consumes them (kept in shared memory, one per warp). */
struct FeedState {
    const uint8_t* src; /* next unit */
    int p;              /* its phase */
    int run;            /* units left in the current run (consecutive k-blocks of one tile) */
    int left;           /* units of the warp's range in phase p after the current run */
    int it;             /* CTA-local tile index of the current run */
    int slot;           /* ring slot of the next unit */
    uint32_t bytes;     /* unit size of the current run */
};

struct TkLayout {
    size_t ring, full, scratch, zero, outbox, tcnt, best, misc, feed, args, args_stride, fdesc, total;
};

/* n_slots is per warp; n_feed matvec phases have a weight-stream descriptor. */
__host__ __device__ inline TkLayout tk_layout(int n_slots, int slot_bytes, size_t scratch_bytes, int n_feed)
{
    TkLayout L;
    L.ring = 0;
    L.full = L.ring + (size_t)NW * n_slots * slot_bytes;
    L.scratch = (L.full + (size_t)NW * n_slots * 8 + 127) & ~(size_t)127;
    L.zero = L.scratch + ((scratch_bytes + 15) & ~(size_t)15);
    L.outbox = L.zero + FL_XENC_ZERO_BYTES;          /* [NW][2][16] floats */
    L.tcnt = L.outbox + (size_t)NW * 2 * 16 * 4;     /* [TCNT] ints */
    L.best = L.tcnt + (size_t)TCNT * 4;              /* [NW][2] */
    L.misc = L.best + NW * 8;                        /* 64 floats */
    L.feed = (L.misc + 64 * 4 + 15) & ~(size_t)15;   /* [NW] FeedState */
    L.args = L.feed + ((NW * sizeof(FeedState) + 15) & ~(size_t)15); /* staged phase arguments */
    const size_t args = sizeof(FlMvArgs) > sizeof(FlAttnArgs) ? sizeof(FlMvArgs) : sizeof(FlAttnArgs);
    L.args_stride = (args + 15) / 16 * 16;           /* two buffers: phases alternate */
    L.fdesc = (L.args + 2 * L.args_stride + 127) & ~(size_t)127; /* [n_feed] FlFeedPhase */
    L.total = L.fdesc + (size_t)n_feed * sizeof(FlFeedPhase);
    return L;
}

__device__ __forceinline__ void consumer_sync() { __syncthreads(); }

__device__ __forceinline__ int ld_acquire(const int* p)
{
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

/* All CTAs finish phase k before any starts phase k+1.  Thread 0 arrives with
 * a release reduction (cumulative over the CTA's writes, ordered before it by
 * the CTA barrier) and polls with acquire loads.  Bounded: gives up after
 * ~2 s, records a timeout and lets the kernel run to its end. */
__device__ void grid_sync(int* bar, int target, int* err, uint64_t* done_stamp)
{
    consumer_sync();
    if (threadIdx.x == 0) {
        if (done_stamp) *done_stamp = fl_globaltimer();
        asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(bar) : "memory");
        if (ld_acquire(bar) < target && !fl_err_set(err)) {
            const uint64_t t0 = fl_globaltimer();
            for (uint32_t it = 0;; it++) {
                if (ld_acquire(bar) >= target) break;
                if (it > 256) __nanosleep(32);
                if ((it & 255u) == 0) {
                    if (fl_err_set(err)) break;
                    if (fl_globaltimer() - t0 > 2000000000ull || it > (1u << 26)) {
                        atomicExch(err, FL_DEV_ERR_TIMEOUT);
                        break;
                    }
                }
            }
        }
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

/* Copies a phase's argument block into shared memory (read there by the hot
 * loops); published by the barrier that follows. */
__device__ __forceinline__ void copy_words(void* dst, const void* src, size_t bytes)
{
    const int n = (int)(bytes / 4);
    for (int i = threadIdx.x; i < n; i += NC)
        reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
}

/* The CTA's U units of a phase (tile-major: unit i = tile i / n_kb, k-block
 * i % n_kb) split into NW contiguous ranges, the first `rem` of length q+1. */
struct Split {
    int q, rem;
    __device__ __forceinline__ int lo(int w) const { return w * q + (w < rem ? w : rem); }
    __device__ __forceinline__ int len(int w) const { return q + (w < rem ? 1 : 0); }
    /* the warp whose range holds unit i */
    __device__ __forceinline__ int owner(int i) const
    {
        const int big = rem * (q + 1);
        return i < big ? i / (q + 1) : rem + (q > 0 ? (i - big) / q : 0);
    }
};

/* 8 consecutive floats p[base .. base+8) (zero beyond n), one vector load
 * pair when they are all in range: through L2 (data written by an earlier
 * phase) or through the read-only path (weights). */
__device__ __forceinline__ void load8_cg(const float* p, int base, int n, float (&o)[8])
{
    if (base + 8 <= n) {
        const float4 u = __ldcg(reinterpret_cast<const float4*>(p + base));
        const float4 v = __ldcg(reinterpret_cast<const float4*>(p + base) + 1);
        o[0] = u.x; o[1] = u.y; o[2] = u.z; o[3] = u.w;
        o[4] = v.x; o[5] = v.y; o[6] = v.z; o[7] = v.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = base + i < n ? __ldcg(p + base + i) : 0.0f;
    }
}

__device__ __forceinline__ void load8(const float* p, int base, int n, float (&o)[8])
{
    if (base + 8 <= n) {
        const float4 u = __ldg(reinterpret_cast<const float4*>(p + base));
        const float4 v = __ldg(reinterpret_cast<const float4*>(p + base) + 1);
        o[0] = u.x; o[1] = u.y; o[2] = u.z; o[3] = u.w;
        o[4] = v.x; o[5] = v.y; o[6] = v.z; o[7] = v.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = base + i < n ? __ldg(p + base + i) : 0.0f;
    }
}

/* 8 consecutive floats of a shared-memory vector (zero beyond n). */
__device__ __forceinline__ void load8_smem(const float* p, int base, int n, float (&o)[8])
{
    if (base + 8 <= n) {
        const float4 u = *reinterpret_cast<const float4*>(p + base);
        const float4 v = *reinterpret_cast<const float4*>(p + base + 4);
        o[0] = u.x; o[1] = u.y; o[2] = u.z; o[3] = u.w;
        o[4] = v.x; o[5] = v.y; o[6] = v.z; o[7] = v.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = base + i < n ? p[base + i] : 0.0f;
    }
}

/* The input of a phase after a row-parallel projection (Wo, down): the
 * projection's rows arrive as (float bits, tag) words in this rank's receive
 * slots, one slot per rank (one on one GPU).  Every thread waits for its
 * element pairs of every rank to carry `tag` — 16-byte loads of two 8-byte
 * words, each word written by one 8-byte store, re-read until current — and
 * sums them in rank order into the shared stage; then x + sum for a plain
 * norm (CTA 0 also stores it in resid_out, the residual stream of later
 * phases), the sum itself for Gemma's pending post-norm input.  Bounded: ~2 s,
 * then FL_DEV_ERR_TIMEOUT; no wait once an error is recorded.  K is even. */
__device__ void stage_parts(const FlMvArgs& a, float* stage, uint32_t tag, int* err)
{
    constexpr int JB = 4; /* element pairs per thread and batch */
    constexpr int QB = 2; /* ranks per poll */
    const int npairs = a.K >> 1;
    const size_t qstride = (size_t)a.part_stride >> 1; /* in pairs */
    const ulonglong2* base = reinterpret_cast<const ulonglong2*>(a.parts);
    const bool add_x = a.in_mode != FL_IN_GEMMA_RESID;
    uint64_t t0 = 0;
    bool timed = false;
    for (int p0 = threadIdx.x; p0 < npairs; p0 += NC * JB) {
        /* the residual pairs first: their load overlaps the wait for the words */
        float2 xr[JB];
#pragma unroll
        for (int j = 0; j < JB; j++) {
            const int pr = p0 + j * NC;
            xr[j] = add_x && pr < npairs ? __ldcg(reinterpret_cast<const float2*>(a.x) + pr) : make_float2(0.0f, 0.0f);
        }
        float2 acc[JB];
        for (int q0 = 0; q0 < a.tp_parts; q0 += QB) {
            ulonglong2 w[QB][JB];
#pragma unroll
            for (int qq = 0; qq < QB; qq++)
#pragma unroll
                for (int j = 0; j < JB; j++) {
                    const int pr = p0 + j * NC;
                    if (q0 + qq < a.tp_parts && pr < npairs) w[qq][j] = fl_ld_volatile_u64x2(base + (q0 + qq) * qstride + pr);
                    else w[qq][j] = make_ulonglong2((unsigned long long)tag << 32, (unsigned long long)tag << 32);
                }
            for (uint32_t it = 0;; it++) {
                bool ok = true;
#pragma unroll
                for (int qq = 0; qq < QB; qq++)
#pragma unroll
                    for (int j = 0; j < JB; j++)
                        if ((uint32_t)(w[qq][j].x >> 32) != tag || (uint32_t)(w[qq][j].y >> 32) != tag) {
                            ok = false;
                            w[qq][j] = fl_ld_volatile_u64x2(base + (q0 + qq) * qstride + p0 + j * NC);
                        }
                if (ok || fl_err_set(err)) break;
                __nanosleep(64); /* every CTA polls the whole vector: keep the re-reads sparse */
                if ((it & 63u) == 0) {
                    const uint64_t now = fl_globaltimer();
                    if (!timed) {
                        t0 = now;
                        timed = true;
                    } else if (now - t0 > 2000000000ull) {
                        atomicExch(err, FL_DEV_ERR_TIMEOUT);
                        break;
                    }
                }
            }
            /* rank order: acc = w[rank 0], then + w[rank 1], ... */
#pragma unroll
            for (int qq = 0; qq < QB; qq++)
#pragma unroll
                for (int j = 0; j < JB; j++) {
                    if (q0 + qq >= a.tp_parts) continue;
                    const float v0 = __uint_as_float((uint32_t)w[qq][j].x), v1 = __uint_as_float((uint32_t)w[qq][j].y);
                    if (q0 + qq == 0) acc[j] = make_float2(v0, v1);
                    else acc[j] = make_float2(__fadd_rn(acc[j].x, v0), __fadd_rn(acc[j].y, v1));
                }
        }
#pragma unroll
        for (int j = 0; j < JB; j++) {
            const int pr = p0 + j * NC;
            if (pr >= npairs) continue;
            float2 v = acc[j];
            if (add_x) {
                v = make_float2(__fadd_rn(xr[j].x, v.x), __fadd_rn(xr[j].y, v.y));
                if (blockIdx.x == 0) reinterpret_cast<float2*>(a.resid_out)[pr] = v;
            }
            reinterpret_cast<float2*>(stage)[pr] = v;
        }
    }
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

template <int PER>
__device__ __forceinline__ void load_row(const float* p, float (&v)[PER])
{
    if constexpr (PER == 2) {
        const float2 a = __ldcg(reinterpret_cast<const float2*>(p));
        v[0] = a.x;
        v[1] = a.y;
    } else {
#pragma unroll
        for (int i = 0; i < PER; i += 4) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(p + i));
            v[i] = a.x;
            v[i + 1] = a.y;
            v[i + 2] = a.z;
            v[i + 3] = a.w;
        }
    }
}

template <int PER>
__device__ __forceinline__ void load_row_smem(const float* p, float (&v)[PER])
{
    if constexpr (PER == 2) {
        const float2 a = *reinterpret_cast<const float2*>(p);
        v[0] = a.x;
        v[1] = a.y;
    } else {
#pragma unroll
        for (int i = 0; i < PER; i += 4) {
            const float4 a = *reinterpret_cast<const float4*>(p + i);
            v[i] = a.x;
            v[i + 1] = a.y;
            v[i + 2] = a.z;
            v[i + 3] = a.w;
        }
    }
}

/* Attention for items (kv head, split) b, b+G, ... in one pass over the
 * item's keys.  A warp takes KPW = 1024/head_dim keys per round: head_dim/32
 * lanes per key form the scores of every query head of the group, then every
 * lane owns head_dim/32 dims of the round's values (loaded once the key
 * registers are free).  Each warp keeps a running (max, sum, output) per
 * query head, updated once per round (online softmax); the CTA merges its
 * warps in warp order into the item's partial (max, sum, unnormalized
 * output), which the combine phase merges across splits.
 * ComputeAttention: LlamaForwardPass.cs:158-211; MistralForwardPass.cs:186-240;
 * Gemma2ForwardPass.cs:126-185. */
template <int HD, int GMAX>
__device__ void phase_attn_t(const FlAttnArgs& a, int pos, float* scr, uint64_t* stamps)
{
    /* profiling: CTA 0 records the end of each step of its first item */
#define FL_STAMP(i) \
    if (stamps && threadIdx.x == 0 && item == (int)blockIdx.x) stamps[i] = fl_globaltimer()
    const int grp = a.n_heads / a.n_kv; /* query heads per kv head, <= GMAX */
    constexpr int LPK = HD / 32;        /* lanes per key for the scores, 8 float4 chunks each */
    constexpr int KPW = 32 / LPK;       /* keys per warp per round */
    constexpr int PER = HD / 32;        /* value dims per lane */
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = lane % LPK, kj = lane / LPK;
    const int kv_dim = a.n_kv * HD;
    float* sq = scr;                   /* [grp][HD] */
    float* sacc = sq + grp * HD;       /* [NW][grp][HD] */
    float* sml = sacc + NW * grp * HD; /* [NW][GMAX][2] running (max, sum) */
    const int seq = pos + 1;
    int start = 0;
    if (a.window < seq) start = seq - a.window;
    const int per = (seq - start + a.n_split - 1) / a.n_split;
    const float inv_cap = a.softcap > 0.0f ? 1.0f / a.softcap : 0.0f;
    const int n_items = a.n_kv * a.n_split;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int kvh = item / a.n_split, split = item % a.n_split;
        const int k0 = start + split * per;
        const int n = max(0, min(seq, k0 + per) - k0);
        const float* kbase = a.k_cache + (size_t)k0 * kv_dim + (size_t)kvh * HD;
        const float* vbase = a.v_cache + (size_t)k0 * kv_dim + (size_t)kvh * HD + lane * PER;
        for (int i = threadIdx.x; i < grp * HD; i += NC) sq[i] = __ldcg(a.q + (size_t)kvh * grp * HD + i);
        consumer_sync();
        FL_STAMP(0);

        float m_run[GMAX], l_run[GMAX], o[GMAX][PER];
#pragma unroll
        for (int h = 0; h < GMAX; h++) {
            m_run[h] = -INFINITY;
            l_run[h] = 0.0f;
#pragma unroll
            for (int p = 0; p < PER; p++) o[h][p] = 0.0f;
        }
        for (int base = warp * KPW; base < n; base += NW * KPW) {
            const bool valid = base + kj < n;
            float sc[GMAX];
#pragma unroll
            for (int h = 0; h < GMAX; h++) sc[h] = 0.0f;
            float4 kv[8]; /* this lane's 8 float4 of key base + kj */
            {
                const float4* kr = reinterpret_cast<const float4*>(kbase + (size_t)min(base + kj, n - 1) * kv_dim);
#pragma unroll
                for (int c = 0; c < 8; c++) kv[c] = __ldcg(kr + c * LPK + qd);
            }
#pragma unroll
            for (int c = 0; c < 8; c++)
#pragma unroll
                for (int h = 0; h < GMAX; h++) {
                    if (h >= grp) break;
                    const float4 q4 = reinterpret_cast<const float4*>(sq + h * HD)[c * LPK + qd];
                    sc[h] = fmaf(q4.x, kv[c].x, sc[h]);
                    sc[h] = fmaf(q4.y, kv[c].y, sc[h]);
                    sc[h] = fmaf(q4.z, kv[c].z, sc[h]);
                    sc[h] = fmaf(q4.w, kv[c].w, sc[h]);
                }
            float vv[KPW][PER]; /* this lane's dims of the round's values */
#pragma unroll
            for (int j = 0; j < KPW; j++) load_row<PER>(vbase + (size_t)min(base + j, n - 1) * kv_dim, vv[j]);
#pragma unroll
            for (int h = 0; h < GMAX; h++) {
                if (h >= grp) break;
#pragma unroll
                for (int off = 1; off < LPK; off <<= 1) sc[h] += __shfl_xor_sync(0xffffffffu, sc[h], off);
                float v = __fmul_rn(sc[h], a.scale);
                if (a.softcap > 0.0f) v = __fmul_rn(tanhf(__fmul_rn(v, inv_cap)), a.softcap);
                v = valid ? v : -INFINITY;
                float mr = v; /* the round's max (key `base` is valid) */
#pragma unroll
                for (int off = LPK; off < 32; off <<= 1) mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, off));
                const float m_new = fmaxf(m_run[h], mr);
                const float corr = __expf(m_run[h] - m_new); /* 0 on the first round */
                const float pw = __expf(v - m_new);          /* 0 past the item's keys */
                m_run[h] = m_new;
                l_run[h] *= corr;
#pragma unroll
                for (int p = 0; p < PER; p++) o[h][p] *= corr;
#pragma unroll
                for (int j = 0; j < KPW; j++) {
                    const float pj = __shfl_sync(0xffffffffu, pw, j * LPK);
                    l_run[h] += pj;
#pragma unroll
                    for (int p = 0; p < PER; p++) o[h][p] = fmaf(pj, vv[j][p], o[h][p]);
                }
            }
        }
        FL_STAMP(1);
#pragma unroll
        for (int h = 0; h < GMAX; h++) {
            if (h >= grp) break;
#pragma unroll
            for (int p = 0; p < PER; p++) sacc[(warp * grp + h) * HD + lane * PER + p] = o[h][p];
            if (lane == 0) {
                sml[(warp * GMAX + h) * 2] = m_run[h];
                sml[(warp * GMAX + h) * 2 + 1] = l_run[h];
            }
        }
        consumer_sync();
        FL_STAMP(2);
        /* the warps, in warp order, into the item's partial */
        float* part = a.part + (size_t)item * grp * (HD + 2);
        for (int i = threadIdx.x; i < grp * HD; i += NC) {
            const int h = i / HD, d = i % HD;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NW; w++) M = fmaxf(M, sml[(w * GMAX + h) * 2]);
            float O = 0.0f, L = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; w++) {
                const float mw = sml[(w * GMAX + h) * 2];
                const float f = mw == -INFINITY ? 0.0f : __expf(mw - M);
                O = fmaf(sacc[(w * grp + h) * HD + d], f, O);
                L = fmaf(sml[(w * GMAX + h) * 2 + 1], f, L);
            }
            part[h * (HD + 2) + 2 + d] = O;
            if (d == 0) {
                part[h * (HD + 2)] = M;
                part[h * (HD + 2) + 1] = L;
            }
        }
        consumer_sync(); /* the item's shared memory is reused by the next item */
        FL_STAMP(3);
    }
#undef FL_STAMP
}

/* The combine phase: query head hq's output from its splits' partials (one
 * CTA per query head, NC/HD threads per output element, split order kept),
 * plus the |max| the next projection's encoding needs. */
template <int HD, int GMAX>
__device__ void phase_attn_combine(const FlAttnArgs& a, float* scr)
{
    constexpr int TPO = NC / HD; /* threads per output dim */
    const int grp = a.n_heads / a.n_kv, S = a.n_split;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t sstride = (size_t)grp * (HD + 2);
    float* w_s = scr;             /* [S] split weights, [S] = total weight */
    float* red = scr + S + 1;     /* [TPO][HD] */
    for (int hq = blockIdx.x; hq < a.n_heads; hq += gridDim.x) {
        const int kvh = hq / grp, h = hq % grp;
        const float* base = a.part + ((size_t)kvh * S * grp + h) * (HD + 2);
        /* this thread's outputs of its first PRE splits, loaded before the
         * split weights exist (they overlap warp 0's work below) */
        constexpr int PRE = 8;
        const int d = threadIdx.x % HD, j = threadIdx.x / HD;
        float ov_pre[PRE];
#pragma unroll
        for (int u = 0; u < PRE; u++) {
            const int sp = j + u * TPO;
            ov_pre[u] = sp < S ? __ldcg(base + sp * sstride + 2 + d) : 0.0f;
        }
        if (warp == 0 && S <= 32) {
            /* one split per lane: its (M, L) loaded once, together */
            const float ms = lane < S ? __ldcg(base + lane * sstride) : -INFINITY;
            const float ls = lane < S ? __ldcg(base + lane * sstride + 1) : 0.0f;
            const float M = fl_warp_max(ms);
            const float f = ms == -INFINITY ? 0.0f : expf(ms - M);
            if (lane < S) w_s[lane] = f;
            const float L = fl_warp_sum(fmaf(ls, f, 0.0f));
            if (lane == 0) w_s[S] = L;
        } else if (warp == 0) {
            float M = -INFINITY;
            for (int s = lane; s < S; s += 32) M = fmaxf(M, __ldcg(base + s * sstride));
            M = fl_warp_max(M);
            float L = 0.0f;
            for (int s = lane; s < S; s += 32) {
                const float ms = __ldcg(base + s * sstride);
                const float f = ms == -INFINITY ? 0.0f : expf(ms - M);
                w_s[s] = f;
                L = fmaf(__ldcg(base + s * sstride + 1), f, L);
            }
            L = fl_warp_sum(L);
            if (lane == 0) w_s[S] = L;
        }
        consumer_sync();
        float O = 0.0f;
#pragma unroll
        for (int u = 0; u < PRE; u++) {
            const int sp = j + u * TPO;
            if (sp < S) O = fmaf(ov_pre[u], w_s[sp], O);
        }
        for (int sp = j + PRE * TPO; sp < S; sp += TPO) O = fmaf(__ldcg(base + sp * sstride + 2 + d), w_s[sp], O);
        red[j * HD + d] = O;
        consumer_sync();
        float amax = 0.0f;
        if (j == 0) {
            float t = 0.0f;
#pragma unroll
            for (int q = 0; q < TPO; q++) t += red[q * HD + d];
            const float L = w_s[S];
            const float ov = L > 0.0f ? t / L : 0.0f;
            a.out[(size_t)hq * HD + d] = ov;
            amax = fabsf(ov);
        }
        amax = fl_warp_max(amax);
        if (lane == 0 && warp * 32 < HD) atomicMax(reinterpret_cast<int*>(a.out_absmax), __float_as_int(amax));
        consumer_sync(); /* w_s and red are reused by the next head */
    }
}

/* Asks L2 for the cached keys and values the CTA's attention items will read
 * (every position before the current one; the current row is written by the
 * QKV phase), so that the attention phase reads them from L2.  Same item
 * split as phase_attn_t. */
__device__ void prefetch_attn_kv(const FlAttnArgs& a, int pos)
{
    const int seq = pos + 1;
    int start = 0;
    if (a.window < seq) start = seq - a.window;
    const int per = (seq - start + a.n_split - 1) / a.n_split;
    const int kv_dim = a.n_kv * a.head_dim;
    const uint32_t row_bytes = (uint32_t)a.head_dim * 4;
    for (int item = blockIdx.x; item < a.n_kv * a.n_split; item += gridDim.x) {
        const int kvh = item / a.n_split, split = item % a.n_split;
        const int k0 = start + split * per, k1 = min(pos, k0 + per);
        for (int i = threadIdx.x; i < 2 * (k1 - k0); i += NC) {
            const float* base = (i & 1) ? a.v_cache : a.k_cache;
            fl_prefetch_l2(base + (size_t)(k0 + (i >> 1)) * kv_dim + (size_t)kvh * a.head_dim, row_bytes);
        }
    }
}

/* ── tensor parallelism ─────────────────────────────────────────────────── */

/* L2 prefetch of a matvec phase's norm weights (and Gemma's pending
 * post-norm weights), whole 16-byte granules. */
__device__ void prefetch_prologue(const FlPhase& ph)
{
    if (ph.kind != FL_PH_MATVEC) return;
    const FlMvArgs& a = ph.mv;
    if (a.in_mode == FL_IN_PLAIN) return;
    const uint32_t bytes = (uint32_t)((a.K * 4 + 15) & ~15);
    if (a.norm_w && (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0) fl_prefetch_l2(a.norm_w, bytes);
    if (a.in_mode == FL_IN_GEMMA_RESID && a.pend_w && (reinterpret_cast<uintptr_t>(a.pend_w) & 15) == 0)
        fl_prefetch_l2(a.pend_w, bytes);
}

/* A warp's private weight ring: S slots of slot_bytes with one full barrier
 * each.  The warp is both producer and consumer of its ring: lane 0 refills a
 * slot once the warp has copied the unit in it to registers. */
struct WarpRing {
    uint8_t* base;
    uint64_t* full;
    int S, slot_bytes;
    const FlFeedPhase* fd; /* the weight-stream descriptors, in shared memory */
};

__device__ __forceinline__ int my_tiles_of(const FlMvArgs& a)
{
    const int G = gridDim.x;
    return a.n_tiles > (int)blockIdx.x ? (a.n_tiles - (int)blockIdx.x + G - 1) / G : 0;
}

/* Moves the cursor to the warp's next run of units: the next tile of its
 * range in the current matvec phase, or the start of its range in the next
 * one (F.p indexes ta.feed, the matvec phases in order).  False once every
 * unit has been issued. */
__device__ __forceinline__ bool feed_advance(const FlTokenArgs& ta, const FlFeedPhase* fd, FeedState& F, int warp)
{
    int kb = 0;
    const FlFeedPhase* fp = fd + (F.p < 0 ? 0 : F.p);
    if (F.left > 0) {
        F.it++;
    } else {
        for (;;) {
            if (F.p + 1 >= ta.n_feed) {
                F.p = ta.n_feed;
                return false;
            }
            F.p++;
            fp = fd + F.p;
            const int G = gridDim.x;
            const int tiles = fp->n_tiles > (int)blockIdx.x ? (fp->n_tiles - (int)blockIdx.x + G - 1) / G : 0;
            const int U = tiles * fp->n_kb;
            const Split S{U / NW, U % NW};
            const int len = S.len(warp);
            if (len == 0) continue;
            const int lo = S.lo(warp);
            F.it = lo / fp->n_kb;
            kb = lo - F.it * fp->n_kb;
            F.left = len;
            break;
        }
    }
    const int n_kb = fp->n_kb;
    const int run = min(n_kb - kb, F.left);
    F.left -= run;
    F.run = run;
    const int tile = (int)blockIdx.x + F.it * (int)gridDim.x;
    const int n_seg = fp->n_seg;
    int t0 = fp->tile0[0], ub = fp->unit_bytes[0];
    const uint8_t* w = fp->w[0];
#pragma unroll
    for (int i = 1; i < FL_MV_MAX_SEG; i++)
        if (i < n_seg && tile >= fp->tile0[i]) {
            t0 = fp->tile0[i];
            ub = fp->unit_bytes[i];
            w = fp->w[i];
        }
    F.bytes = (uint32_t)ub;
    F.src = w + ((size_t)(tile - t0) * n_kb + kb) * F.bytes;
    return true;
}

/* Lane 0: issues the copy of the warp's next unit into the next ring slot. */
__device__ __forceinline__ void feed(const FlTokenArgs& ta, const WarpRing& R, FeedState& F, int warp)
{
    if (F.run == 0 && !feed_advance(ta, R.fd, F, warp)) return;
    const int slot = F.slot;
    const uint32_t bytes = F.bytes;
    const uint8_t* src = F.src;
    fl_mbar_expect_tx(&R.full[slot], bytes);
    fl_bulk_g2s(R.base + (size_t)slot * R.slot_bytes, src, bytes, &R.full[slot]);
    F.src = src + bytes;
    F.run--;
    F.slot = slot + 1 == R.S ? 0 : slot + 1;
}

/* n consecutive units (k-blocks kb0..kb0+n-1 of one tile) of format FMT.  A
 * unit's slot is refilled as soon as its bytes are in registers. */
/* Per-warp counters of a matvec phase (reported for CTA 0 when profiling). */
struct UnitStats {
    uint64_t wait_cycles;
    uint32_t waits, units;
};

template <int FMT, bool EXP>
__device__ __forceinline__ void run_units(const FlTokenArgs& ta, const WarpRing& R, FeedState& f, int& cslot,
                                          uint32_t& cpar, int n, int kb0, const uint8_t* bptr, bool bval,
                                          const uint8_t* zero, const short2* xs, const float* xsum, int lane,
                                          int warp, Acc& A, UnitStats& st)
{
    for (int k = 0; k < n; k++) {
        if (!fl_mbar_test(&R.full[cslot], cpar)) {
            const long long t0 = clock64();
            fl_mbar_wait(&R.full[cslot], cpar, ta.err);
            st.wait_cycles += (uint64_t)(clock64() - t0);
            st.waits++;
        }
        st.units++;
        const int kb = kb0 + k;
        process_unit<FMT, EXP>(R.base + (size_t)cslot * R.slot_bytes, kb, unit_bptr(bptr, bval, zero, kb), xs, xsum,
                               lane, A, [&]() {
                                   __syncwarp();
                                   if (lane == 0) {
                                       fl_fence_proxy_async();
                                       feed(ta, R, f, warp);
                                   }
                               });
        if (++cslot == R.S) {
            cslot = 0;
            cpar ^= 1u;
        }
    }
}

template <int HD, int GMAX>
__global__ void __launch_bounds__(NT, 1) fl_token_kernel(const __grid_constant__ FlTokenArgs ta)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const TkLayout Ls = tk_layout(ta.n_slots, ta.slot_bytes, ta.scratch_bytes, ta.n_feed);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int G = gridDim.x;
    const WarpRing R{smem + Ls.ring + (size_t)warp * ta.n_slots * ta.slot_bytes,
                     reinterpret_cast<uint64_t*>(smem + Ls.full) + warp * ta.n_slots, ta.n_slots, ta.slot_bytes,
                     reinterpret_cast<const FlFeedPhase*>(smem + Ls.fdesc)};
    uint8_t* scratch = smem + Ls.scratch;
    uint8_t* zero = smem + Ls.zero;
    float* outbox = reinterpret_cast<float*>(smem + Ls.outbox);
    int* tcnt = reinterpret_cast<int*>(smem + Ls.tcnt);
    float* best = reinterpret_cast<float*>(smem + Ls.best);
    float* misc = reinterpret_cast<float*>(smem + Ls.misc);
    FeedState f; /* lane 0's cursor (registers) */

    f.src = nullptr;
    f.p = -1;
    f.run = f.left = f.it = f.slot = 0;
    f.bytes = 0;
    if (lane == 0)
        for (int i = 0; i < R.S; i++) fl_mbar_init(&R.full[i], 1);
    for (int i = tid; i < TCNT; i += NT) tcnt[i] = 0;
    for (int i = tid; i < FL_XENC_ZERO_BYTES; i += NT) zero[i] = 0;
    /* the lane-0 cursors walk the descriptors at every run boundary: keep them on chip */
    copy_words(smem + Ls.fdesc, ta.feed, (size_t)ta.n_feed * sizeof(FlFeedPhase));
    fl_fence_mbar_init();
    __syncthreads();

    /* the weights do not depend on the step's data: start streaming now */
    if (lane == 0)
        for (int k = 0; k < R.S; k++) feed(ta, R, f, warp);
    int cslot = 0;
    uint32_t cpar = 0;

    float best_v = 0.0f;
    int best_i = 0x7fffffff;
    const int tp_epoch0 = ta.tp_size > 1 ? __ldcg(ta.tp_epoch) : 0;
    /* row exchanges of earlier steps: exchange x of this step carries tag tp_rows0 + x */
    const uint32_t tp_rows0 = ta.tp_epoch ? (uint32_t)__ldcg(ta.tp_epoch + 1) : 0u;
    int n_sync = 0; /* grid barriers passed */
    /* the step's position: every phase of the launch uses the same one (the
     * device-resident loop advances it only after the last phase) */
    const int pos0 = __ldcg(ta.pos);
    /* The warp's k-blocks of a matvec input are kb = warp + r*NW; lane l
     * encodes inputs kb*256 + 8l .. +8.  With up to RK k-blocks per warp every
     * input load of the prologue is issued at once and the values stay in
     * registers until they are encoded. */
    constexpr int RK = 4;
    for (int p = 0; p < ta.n_phases; p++) {
        const int kind = ta.phases[p].kind;
        /* this phase's arguments into the buffer phase p-2 used (every warp
         * passed the barrier after it), published by the barrier below */
        uint8_t* abuf = smem + Ls.args + (size_t)(p & 1) * Ls.args_stride;
        if (kind == FL_PH_MATVEC) {
            copy_words(abuf, &ta.phases[p].mv, sizeof(FlMvArgs));
            if (p + 1 < ta.n_phases && ta.phases[p + 1].kind == FL_PH_ATTN) prefetch_attn_kv(ta.phases[p + 1].at, pos0);
        } else if (kind == FL_PH_ATTN || kind == FL_PH_ATTN_COMBINE) {
            copy_words(abuf, &ta.phases[p].at, sizeof(FlAttnArgs));
        }
        /* The next matvec phase's static prologue operands (norm weights) do
         * not depend on the step's data: one CTA asks L2 for them a phase
         * early, so that the prologue after the barrier finds them there
         * instead of waiting on HBM behind the weight stream. */
        if (p + 1 < ta.n_phases && tid == 0 && (int)blockIdx.x == (p * 7) % G) prefetch_prologue(ta.phases[p + 1]);
        uint64_t* done_stamp = ta.cta_done && p > 0 ? ta.cta_done + (size_t)(p - 1) * G + blockIdx.x : nullptr;
        /* a phase that reads a row exchange waits on the exchange's tags in
         * its prologue instead of at a grid barrier */
        const int xk = ta.phases[p].xk;
        if (p > 0 && xk == 0) {
            grid_sync(ta.bar, ++n_sync * G, ta.err, done_stamp);
        } else {
            if (done_stamp && tid == 0) *done_stamp = fl_globaltimer();
            consumer_sync();
        }
        if (ta.timestamps && blockIdx.x == 0 && tid == 0) ta.timestamps[p] = fl_globaltimer();
        if (kind == FL_PH_EMBED) {
            phase_embed(ta.phases[p].em, ta.err);
            continue;
        }
        if (kind == FL_PH_ATTN) {
            phase_attn_t<HD, GMAX>(*reinterpret_cast<const FlAttnArgs*>(abuf), pos0, reinterpret_cast<float*>(scratch),
                                   ta.detail && blockIdx.x == 0 ? ta.detail + (size_t)p * NW * 4 : nullptr);
            continue;
        }
        if (kind == FL_PH_ATTN_COMBINE) {
            phase_attn_combine<HD, GMAX>(*reinterpret_cast<const FlAttnArgs*>(abuf), reinterpret_cast<float*>(scratch));
            continue;
        }
        /* ── matvec phase ── */
        const FlMvArgs& a = *reinterpret_cast<const FlMvArgs*>(abuf);
        const int n_kb = a.n_kb;
        uint8_t* xl = scratch;
        const size_t nc = (size_t)n_kb * 8;
        short2* xs = reinterpret_cast<short2*>(scratch + nc * FL_XENC_LIMB_BYTES);
        float* xsum = reinterpret_cast<float*>(scratch + nc * (FL_XENC_LIMB_BYTES + FL_XENC_LSUM_BYTES));
        Prolog P{a.in_mode, a.K, a.x, a.norm_w, a.pend, a.pend_w, 1.0f, 1.0f};
        const bool in_regs = n_kb <= RK * NW;
        float amax;
        if (in_regs) {
            const int mode = a.in_mode;
            float xv[RK][8];
            const float am_plain = mode == FL_IN_PLAIN ? __ldcg(a.absmax) : 0.0f;
            /* tensor parallelism: x + the ranks' partial rows (or Gemma's
             * pending vector) summed once into shared memory, read from there */
            const bool staged = a.tp_parts > 0;
            float* stage = reinterpret_cast<float*>(scratch + ta.scratch_bytes - (size_t)a.K * 4);
            if (staged) {
                stage_parts(a, stage, tp_rows0 + (uint32_t)xk, ta.err);
                consumer_sync();
            }
            if (mode == FL_IN_GEMMA_RESID) {
                float sp = 0.0f, dummy = 0.0f;
                for (int i = tid; i < a.K; i += NC) {
                    const float v = staged ? stage[i] : __ldcg(a.pend + i);
                    sp = fmaf(v, v, sp);
                }
                consumer_sum_max(sp, dummy, misc);
                P.rms_p = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(sp, (float)a.K), 1e-6f));
            }
#pragma unroll
            for (int r = 0; r < RK; r++) {
                const int base = (warp + r * NW) * 256 + lane * 8;
                if (staged && mode != FL_IN_GEMMA_RESID) load8_smem(stage, base, a.K, xv[r]);
                else load8_cg(a.x, base, a.K, xv[r]);
            }
            if (mode == FL_IN_PLAIN) {
                amax = am_plain;
            } else {
                float ss = 0.0f, mx = 0.0f;
#pragma unroll
                for (int r = 0; r < RK; r++) {
                    const int base = (warp + r * NW) * 256 + lane * 8;
                    if (base >= a.K) continue;
                    float w[8];
                    load8(a.norm_w, base, a.K, w);
                    if (mode == FL_IN_GEMMA_RESID) {
                        /* x' = x + GemmaRmsNorm(pend, pend_w), kept by CTA 0 */
                        float pe[8], pw[8];
                        if (staged) load8_smem(stage, base, a.K, pe);
                        else load8_cg(a.pend, base, a.K, pe);
                        load8(a.pend_w, base, a.K, pw);
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            xv[r][i] = __fadd_rn(xv[r][i], __fmul_rn(__fmul_rn(pe[i], P.rms_p), __fadd_rn(pw[i], 1.0f)));
                        if (blockIdx.x == 0)
#pragma unroll
                            for (int i = 0; i < 8; i++)
                                if (base + i < a.K) a.resid_out[base + i] = xv[r][i];
                    }
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const float xi = xv[r][i];
                        const float wi = mode == FL_IN_RMSNORM ? w[i] : __fadd_rn(w[i], 1.0f);
                        ss = fmaf(xi, xi, ss);
                        /* x*w per element; the norm's 1/rms scales it after the
                         * reduction (the 21-bit encoding absorbs the rounding) */
                        xv[r][i] = base + i < a.K ? xi * wi : 0.0f;
                        mx = fmaxf(mx, fabsf(xv[r][i]));
                    }
                }
                consumer_sum_max(ss, mx, misc);
                P.rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)a.K), a.eps));
                amax = P.rms * mx * 1.00001f;
            }
            const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
            const float scale = mode == FL_IN_PLAIN ? 1.0f : P.rms;
#pragma unroll
            for (int r = 0; r < RK; r++) {
                const int kb = warp + r * NW;
                if (kb < n_kb) {
                    float v[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) v[i] = xv[r][i] * scale;
                    encode_values(v, kb, inv, lane, xl, xs, xsum);
                }
            }
        } else {
            /* long inputs: one k-block at a time */
            if (a.in_mode == FL_IN_PLAIN) {
                amax = __ldcg(a.absmax);
            } else {
                float ss = 0.0f, mx = 0.0f;
                if (a.in_mode == FL_IN_GEMMA_RESID) {
                    float sp = 0.0f, dummy = 0.0f;
                    for (int i = tid; i < a.K; i += NC) {
                        const float v = __ldcg(a.pend + i);
                        sp = fmaf(v, v, sp);
                    }
                    consumer_sum_max(sp, dummy, misc);
                    P.rms_p = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(sp, (float)a.K), 1e-6f));
                }
                for (int i = tid; i < a.K; i += NC) {
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
            for (int kb = warp; kb < n_kb; kb += NW) encode_kblock(P, kb, inv, lane, xl, xs, xsum);
        }
        const float xscale = amax / 127.0f;
        consumer_sync();
        const int pos = pos0;
        const int limb = g & 3;
        const bool bval = (limb < 3) && ((g >> 2) == (t >> 1));
        const uint8_t* bptr = xl + (limb * 4 + t) * 8;
        const float wlane = ((t & 1) ? (1.0f / 16384.0f) : 1.0f) * xscale;
        const int Uph = my_tiles_of(a) * n_kb;
        const Split S{Uph / NW, Uph % NW};
        const int lo = S.lo(warp), hi = lo + S.len(warp);
        const int first_it = lo / n_kb, last_it = hi > lo ? (hi - 1) / n_kb : first_it;
        /* the epilogue operands of the range's first and last tile, loaded now */
        const bool has_pre = hi > lo && (a.epi == FL_EPI_RESID || a.epi == FL_EPI_QKV);
        float2 pre0 = make_float2(0.0f, 0.0f), pre1 = pre0;
        if (has_pre) {
            pre0 = epilogue_operand(a, (int)blockIdx.x + first_it * G, lane, pos);
            pre1 = epilogue_operand(a, (int)blockIdx.x + last_it * G, lane, pos);
        }
        UnitStats st{0, 0, 0};
        bool pushed = false; /* this thread stored epilogue rows (to peers, with tensor parallelism) */
        if (ta.detail && blockIdx.x == 0 && tid == 0) ta.detail[(size_t)ta.n_phases * NW * 4 + p] = fl_globaltimer();

        int i0 = lo;
        while (i0 < hi) {
            /* one tile: the units [i0, i1) of this warp's range inside it */
            const int it = i0 / n_kb;
            const int i1 = min(hi, (it + 1) * n_kb);
            const int tile = (int)blockIdx.x + it * G;
            const int si = seg_of(a, tile);
            const FlMvSeg& sg = a.seg[si];
            const int c = i1 - i0, kb0 = i0 - it * n_kb;
            Acc A{0.0f, 0.0f, 0.0f, 0.0f};
#define FL_RUN(F, E) run_units<F, E>(ta, R, f, cslot, cpar, c, kb0, bptr, bval, zero, xs, xsum, lane, warp, A, st)
            if (!sg.expanded && sg.fmt == FL_FMT_Q4K) {
                FL_RUN(FL_FMT_Q4K, false);
            } else if (!sg.expanded && sg.fmt == FL_FMT_Q6K) {
                FL_RUN(FL_FMT_Q6K, false);
            } else if (sg.expanded) {
                switch (sg.fmt) {
                case FL_FMT_Q4K: FL_RUN(FL_FMT_Q4K, true); break;
                case FL_FMT_Q5K: FL_RUN(FL_FMT_Q5K, true); break;
                case FL_FMT_Q6K: FL_RUN(FL_FMT_Q6K, true); break;
                default: FL_RUN(FL_FMT_Q8K, true); break;
                }
            } else {
                switch (sg.fmt) {
                case FL_FMT_Q5K: FL_RUN(FL_FMT_Q5K, false); break;
                case FL_FMT_Q8_0: FL_RUN(FL_FMT_Q8_0, false); break;
                case FL_FMT_Q4_0: FL_RUN(FL_FMT_Q4_0, false); break;
                default: FL_RUN(FL_FMT_Q8K, false); break;
                }
            }
#undef FL_RUN
            i0 = i1;
            float v0 = fmaf(A.res0, wlane, -A.m0), v1 = fmaf(A.res1, wlane, -A.m1);
            v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
            v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
            v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
            v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
            float v;
            if (c == n_kb) {
                /* the whole tile is in this warp: lane r (mod 16) takes row r */
                const float a0 = __shfl_sync(0xffffffffu, v0, (lane & 7) * 4);
                const float a1 = __shfl_sync(0xffffffffu, v1, (lane & 7) * 4);
                v = (lane & 8) ? a1 : a0;
            } else {
                /* a tile shared with the neighbouring range(s): outbox slot 0
                 * holds the partial of the range's first tile, slot 1 its last */
                float* mine = outbox + ((size_t)warp * 2 + (it == first_it ? 0 : 1)) * 16;
                if (t == 0) {
                    mine[g] = v0;
                    mine[g + 8] = v1;
                }
                __threadfence_block();
                __syncwarp();
                int last = 0;
                if (lane == 0) last = atomicAdd(&tcnt[it], c) + c == n_kb;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (!last) continue;
                __threadfence_block();
                const int wa = S.owner(it * n_kb), wb = S.owner((it + 1) * n_kb - 1);
                v = 0.0f;
                for (int w = wa; w <= wb; w++) {
                    const int fw = S.lo(w) / n_kb;
                    const volatile float* ov = outbox + ((size_t)w * 2 + (it == fw ? 0 : 1)) * 16;
                    v += ov[lane & 15];
                }
                if (lane == 0) tcnt[it] = 0;
            }
            epilogue_any(a, sg, si, tile, lane, v, pos, best_v, best_i, it == first_it ? pre0 : pre1,
                         has_pre && (it == first_it || it == last_it), tp_rows0 + (uint32_t)a.push_x);
            pushed |= lane < 16;
        }
        if (ta.detail && blockIdx.x == 0 && lane == 0) {
            uint64_t* d = ta.detail + ((size_t)p * NW + warp) * 4;
            d[0] = fl_globaltimer();
            d[1] = st.wait_cycles;
            d[2] = st.waits;
            d[3] = st.units;
        }
        /* rows pushed to other GPUs are visible system-wide before this CTA
         * reports the phase done (only the lanes that stored them fence) */
        if (a.epi == FL_EPI_LOGITS && a.tp_n > 0 && pushed) __threadfence_system();

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
                    const float bw = best[w * 2];
                    const int iw = __float_as_int(best[w * 2 + 1]);
                    if (iw != 0x7fffffff && (bi == 0x7fffffff || fl_argmax_better(bw, iw, bv, bi))) {
                        bv = bw;
                        bi = iw;
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
                    const float bw = __ldcg(&a.cta_best[b * 2]);
                    const int iw = __float_as_int(__ldcg(&a.cta_best[b * 2 + 1]));
                    if (iw != 0x7fffffff && (bi == 0x7fffffff || fl_argmax_better(bw, iw, bv, bi))) {
                        bv = bw;
                        bi = iw;
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
                if (lane == 0 && ta.tp_size > 1) {
                    /* across ranks: each rank's best, in rank order */
                    for (int q = 0; q < ta.tp_size; q++) {
                        float* bq = reinterpret_cast<float*>(ta.tp_peer[q] + FL_TP_BEST_OFF) + 2 * ta.tp_rank;
                        bq[0] = bv;
                        bq[1] = __int_as_float(bi);
                    }
                    __threadfence_system();
                }
                if (ta.tp_size > 1) {
                    __syncwarp();
                    if (lane == 0) {
                        const int epoch = tp_epoch0 + ta.tp_n_exchanges;
                        for (int q = 0; q < ta.tp_size; q++)
                            fl_st_release_sys(reinterpret_cast<int*>(ta.tp_peer[q] + FL_TP_FLAGS_OFF) + ta.tp_rank,
                                              epoch);
                        const int* fl = reinterpret_cast<const int*>(ta.tp_peer[ta.tp_rank] + FL_TP_FLAGS_OFF);
                        const float* bb = reinterpret_cast<const float*>(ta.tp_peer[ta.tp_rank] + FL_TP_BEST_OFF);
                        const uint64_t t0 = fl_globaltimer();
                        bv = 0.0f;
                        bi = 0x7fffffff;
                        for (int q = 0; q < ta.tp_size; q++) {
                            for (uint32_t it = 0; !fl_err_set(ta.err) && fl_ld_acquire_sys(fl + q) < epoch; it++)
                                if ((it & 255u) == 0 && fl_globaltimer() - t0 > 2000000000ull) {
                                    atomicExch(ta.err, FL_DEV_ERR_TIMEOUT);
                                    break;
                                }
                            const float bw = __ldcg(bb + 2 * q);
                            const int iw = __float_as_int(__ldcg(bb + 2 * q + 1));
                            if (iw != 0x7fffffff && (bi == 0x7fffffff || fl_argmax_better(bw, iw, bv, bi))) {
                                bv = bw;
                                bi = iw;
                            }
                        }
                        *ta.tp_epoch = epoch;
                    }
                }
                if (lane == 0) {
                    *a.argmax_out = bi;
                    *a.counter = 0;
                    if (ta.tp_epoch) ta.tp_epoch[1] = (int32_t)(tp_rows0 + (uint32_t)ta.tp_rows_per_step);
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

/* Kernel of the (head_dim, largest group) instances compiled in this unit. */
template <int HD, int GMAX>
const void* kernel_ptr()
{
    return reinterpret_cast<const void*>(fl_token_kernel<HD, GMAX>);
}

} // namespace
} // namespace fltk

#endif
