/*
 * fl_tc_gemm.cu — the prompt path's and the batched steps' fp16 GEMM on the
 * Blackwell tensor cores (tcgen05), written for sm_100a:
 *
 *   Y[b][n][m] = alpha * sum_k A[b][m][k] * B[b][n][k]  (+ beta * Y[b][n][m])
 *
 * A holds the weight rows (the split-fp16 [hi | hi | lo] rows of a dequantized
 * matrix, or the keys / transposed values of attention), B the activation rows
 * (tokens), both K-major fp16; Y is fp32, one row per token.  This is
 * LinearProjection (src/DotNetFoundryLLM.Architectures/LlamaForwardPass.cs:
 * 237-260) for a chunk of prompt tokens at once, the reference running it one
 * token at a time (LlamaLanguageModel.cs:133-137).
 *
 * Structure (one CTA per SM, persistent over output tiles of 128 weight rows x
 * BN tokens, tiles with the same weight rows adjacent so the CTAs that run at
 * once share them through L2):
 *  - warp 0, one lane: TMA (cp.async.bulk.tensor.2d, 128-byte swizzle, no
 *    multicast) of the A and B tiles of each 64-wide k-block into a ring of
 *    shared-memory stages (full / empty mbarriers);
 *  - warp 1: allocates the tensor memory (two accumulators of BN fp32
 *    columns), one lane issues tcgen05.mma.kind::f16 (M 128, N BN, K 16; four
 *    per stage) and tcgen05.commit frees each stage and, per tile, signals the
 *    accumulator full;
 *  - warps 2-5: the epilogue reads its 32 TMEM lanes (tcgen05.ld 32x32b) and
 *    stores alpha*acc (+beta*Y) with each warp writing 128 contiguous bytes
 *    per token, while the other accumulator takes the next tile's MMAs.
 * Every wait is bounded (~2 s): on expiry the CTA records FL_DEV_ERR_TIMEOUT,
 * stops issuing, waits (bounded) for its copies and MMAs in flight, frees its
 * tensor memory and returns.
 */
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "fl_device.cuh"
#include "fl_kernels.h"

namespace {

constexpr int BM = 128;         /* weight rows per tile (UMMA M) */
constexpr int BK = 64;          /* fp16 per k-block: one 128-byte swizzle row */
constexpr int kThreads = 192;   /* 6 warps */

template <int BN>
struct Cfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
    static constexpr int TMEM_COLS = 2 * BN; /* two accumulators: a power of two >= 32 */
    static constexpr int BAR_BYTES = 256;
    static constexpr size_t SMEM = (size_t)STAGES * STAGE + 1024 + BAR_BYTES;
};

/* Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle
 * layout TMA writes: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO),
 * descriptor version 1 (sm_100), layout type 2 (128-byte swizzle). */
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr)
{
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;             /* LBO: unused for swizzled K-major */
    d |= (uint64_t)(1024 >> 4) << 32;   /* SBO */
    d |= (uint64_t)1 << 46;             /* version */
    d |= (uint64_t)2 << 61;             /* SWIZZLE_128B */
    return d;
}

/* Instruction descriptor of kind::f16: A, B fp16, D fp32, both K-major. */
template <int BN>
__host__ __device__ constexpr uint32_t idesc_f16()
{
    return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(uint32_t sdst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            sdst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(fl_smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum)
{
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}

/* Arrives on `bar` once every tcgen05.mma this thread issued so far completed. */
__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(fl_smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

/* 32 lanes x 32 consecutive fp32 columns of the accumulator: thread t of the
 * warp gets lane (32*quarter + t), columns col..col+31. */
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct TcArgs {
    int M, N, K, batch;            /* per batch: M weight rows, N tokens, K */
    int a_batch_rows, b_batch_rows; /* rows of A / B between batches in the 2-D maps */
    int mt, nt, ks;                /* tiles per batch along M and N; K splits */
    float* Y;
    long long ldy, y_batch;        /* Y row stride and batch stride (elements) */
    float alpha, beta;
    float* part;                   /* ks > 1: [ks][batch][N][M] partial products */
    int causal, c_grp, c_start, c_seg, c_seglen; /* see FlTcGemm */
    int* err;
};

/* The output tile of work item t (split s fastest, then token tiles, then
 * weight-row tiles, then batches) and its k-blocks: k-block i of the tile is
 * global k-block kb_of(i), i < count.  Causal mode 1 gives a count of 0 to a
 * tile whose A rows (keys) all lie past the last key any of its B rows (query
 * rows of tokens start..) may attend to; mode 2 keeps, of each of the c_seg
 * segments of c_seglen columns of K, the columns (keys) below that bound. */
struct TileWork {
    int b, m0, n0, s;
    int count, kb_lo, per_seg, seg_kb;
    __device__ __forceinline__ int kb_of(int i) const
    {
        return per_seg ? (i / per_seg) * seg_kb + (i % per_seg) : kb_lo + i;
    }
};

template <int BN>
__device__ __forceinline__ TileWork tile_work(const TcArgs& g, int t, int nkb)
{
    TileWork w;
    w.s = t % g.ks;
    const int r0 = t / g.ks;
    w.b = r0 / (g.mt * g.nt);
    const int r = r0 % (g.mt * g.nt);
    w.m0 = (r / g.nt) * BM;
    w.n0 = (r % g.nt) * BN;
    w.kb_lo = (int)((long long)nkb * w.s / g.ks);
    w.count = (int)((long long)nkb * (w.s + 1) / g.ks) - w.kb_lo;
    w.per_seg = 0;
    w.seg_kb = 0;
    if (g.causal) {
        const int last_row = min(g.N, w.n0 + BN) - 1;
        const int kbound = g.c_start + last_row / g.c_grp + 1; /* keys [0, kbound) */
        if (g.causal == 1) {
            if (w.m0 >= kbound) w.count = 0;
        } else {
            const int kmax = min(g.c_seglen, kbound);
            w.seg_kb = g.c_seglen / BK;
            w.per_seg = (kmax + BK - 1) / BK;
            w.count = w.per_seg * g.c_seg;
            w.kb_lo = 0;
        }
    }
    return w;
}

/* Bounded wait on an mbarrier phase; false (and the CTA's abort flag and the
 * launch's error set) once ~2 s passed or another role of the CTA gave up. */
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err)
{
    if (fl_mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = fl_globaltimer();
    for (uint32_t it = 1;; it++) {
        if (fl_mbar_try_wait(bar, parity)) return true;
        if ((it & 1023u) == 0) {
            if (*abort) return false;
            if (fl_globaltimer() - t0 > 2000000000ull) {
                *abort = 1;
                if (err) atomicExch(err, FL_DEV_ERR_TIMEOUT);
                return false;
            }
        }
    }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    fl_tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                      const TcArgs g)
{
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    /* 128-byte swizzled TMA destinations want 1024-byte alignment */
    const uint32_t raw_u32 = fl_smem_u32(smem_raw);
    const uint32_t pad = ((raw_u32 + 1023u) & ~1023u) - raw_u32;
    uint8_t* smem = smem_raw + pad;
    const uint32_t s_base = raw_u32 + pad;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)C::STAGES * C::STAGE);
    uint64_t* empty = full + C::STAGES;
    uint64_t* tfull = empty + C::STAGES;   /* [2] accumulator ready for the epilogue */
    uint64_t* tempty = tfull + 2;          /* [2] accumulator drained by the epilogue */
    uint64_t* done = tempty + 2;           /* MMA drain after an abort */
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
    volatile int* consumed = reinterpret_cast<volatile int*>(tmem_holder + 2); /* k-blocks the MMA lane took */

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = g.batch * g.mt * g.nt * g.ks;
    const int nkb = (g.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            fl_mbar_init(&full[s], 1);
            fl_mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            fl_mbar_init(&tfull[a], 1);
            fl_mbar_init(&tempty[a], 4); /* one arrival per epilogue warp */
        }
        fl_mbar_init(done, 1);
        *abort = 0;
        *consumed = 0;
        fl_fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(fl_smem_u32(tmem_holder)),
                     "r"(C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    int issued = 0; /* producer: k-blocks loaded */
    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const TileWork w = tile_work<BN>(g, t, nkb);
                const int arow = w.b * g.a_batch_rows + w.m0;
                const int brow = w.b * g.b_batch_rows + w.n0;
                for (int i = 0; i < w.count; i++, issued++) {
                    const int kb = w.kb_of(i);
                    const int s = issued % C::STAGES;
                    if (issued >= C::STAGES && !tc_wait(&empty[s], ((issued / C::STAGES) - 1) & 1, abort, g.err)) {
                        ok = false;
                        break;
                    }
                    fl_mbar_expect_tx(&full[s], C::STAGE);
                    const uint32_t sa = s_base + (uint32_t)(s * C::STAGE);
                    tma_load_2d(sa, &map_a, kb * BK, arow, &full[s]);
                    tma_load_2d(sa + C::A_BYTES, &map_b, kb * BK, brow, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16<BN>();
            bool ok = true;
            int kcount = 0, local = 0;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const TileWork w = tile_work<BN>(g, t, nkb);
                if (w.count == 0) continue; /* no MMA, no epilogue */
                const int acc = local & 1;
                if (local >= 2 && !tc_wait(&tempty[acc], ((local >> 1) - 1) & 1, abort, g.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                for (int i = 0; i < w.count; i++, kcount++) {
                    const int s = kcount % C::STAGES;
                    if (!tc_wait(&full[s], (kcount / C::STAGES) & 1, abort, g.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = s_base + (uint32_t)(s * C::STAGE);
                    const uint64_t da = umma_desc_sw128(sa), db = umma_desc_sw128(sa + C::A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; k++) /* K 16 = 32 bytes: +2 in 16-byte units */
                        umma_f16(d, da + 2 * k, db + 2 * k, idesc, (i | k) != 0);
                    umma_commit(&empty[s]);
                    *consumed = kcount + 1;
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
                local++;
            }
            /* every MMA issued has completed before the tensor memory is freed */
            umma_commit(done);
            bool dummy = fl_mbar_wait(done, 0, nullptr);
            (void)dummy;
        }
    } else {
        /* epilogue: warps 2..5 own TMEM lanes 32*(warp % 4) .. +31 */
        const int q = warp & 3;
        int local = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
            const TileWork w = tile_work<BN>(g, t, nkb);
            if (w.count == 0) continue;
            const int acc = local & 1;
            if (!tc_wait(&tfull[acc], (local >> 1) & 1, abort, g.err)) break;
            local++;
            tc_fence_after();
            const int m = w.m0 + q * 32 + lane;
            const int n0 = w.n0;
            /* a K split writes its raw partial; the reduction applies alpha, beta */
            const bool split = g.ks > 1;
            float* yb = split ? g.part + ((long long)w.s * g.batch + w.b) * g.N * (long long)g.M
                              : g.Y + (long long)w.b * g.y_batch;
            const long long ldy = split ? g.M : g.ldy;
#pragma unroll 1
            for (int c = 0; c < BN / 32; c++) {
                uint32_t v[32];
                tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), v);
                if (m < g.M) {
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const int n = n0 + c * 32 + j;
                        if (n < g.N) {
                            float* p = yb + (long long)n * ldy + m;
                            if (split) {
                                *p = __uint_as_float(v[j]);
                            } else {
                                float o = g.alpha * __uint_as_float(v[j]);
                                if (g.beta != 0.0f) o = fmaf(g.beta, *p, o);
                                *p = o;
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) fl_mbar_arrive(&tempty[acc]);
        }
    }

    __syncthreads();
    if (warp == 0 && lane == 0 && *abort) {
        /* copies issued but never consumed land before the CTA's memory goes */
        for (int i = *consumed; i < issued; i++) {
            bool dummy = fl_mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1, nullptr);
            (void)dummy;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::TMEM_COLS)
                     : "memory");
    }
}

/* Y = alpha * (sum of the K splits' partials, in split order) + beta * Y. */
__global__ void split_reduce_kernel(const float* __restrict__ part, int ks, int batch, int N, int M, float* Y,
                                    long long ldy, long long y_batch, float alpha, float beta)
{
    const long long per = (long long)N * M, count = per * batch;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count; i += (long long)gridDim.x * blockDim.x) {
        float sum = part[i];
        for (int s = 1; s < ks; s++) sum += part[(long long)s * count + i];
        const long long b = i / per, r = i % per, n = r / M, m = r % M;
        float* p = Y + b * y_batch + n * ldy + m;
        float o = alpha * sum;
        if (beta != 0.0f) o = fmaf(beta, *p, o);
        *p = o;
    }
}

/* cuTensorMapEncodeTiled from the driver, looked up once. */
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

/* A 2-D K-major fp16 map: `rows` rows of K elements, `ld` elements apart,
 * boxes of 64 x box_rows with 128-byte swizzle; outside the matrix reads 0. */
cudaError_t make_map(CUtensorMap* map, const __half* base, long long rows, int K, long long ld, int box_rows)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) || ((ld * 2) & 15) || K <= 0 || rows <= 0)
        return cudaErrorInvalidValue;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

int g_sm_count[64];

template <int BN>
cudaError_t launch(const __half* A, long long lda, const __half* B, long long ldb, const FlTcGemm& p, cudaStream_t st)
{
    using C = Cfg<BN>;
    static bool configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(fl_tc_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
        if (e != cudaSuccess) return e;
        if (!g_sm_count[dev]) {
            e = cudaDeviceGetAttribute(&g_sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess) return e;
        }
        configured[dev] = true;
    }
    TcArgs g;
    g.M = p.M;
    g.N = p.N;
    g.K = p.K;
    g.batch = p.batch;
    g.a_batch_rows = p.a_batch_rows;
    g.b_batch_rows = p.b_batch_rows;
    g.mt = (p.M + BM - 1) / BM;
    g.nt = (p.N + BN - 1) / BN;
    g.ks = p.ksplit > 1 ? p.ksplit : 1;
    g.Y = p.Y;
    g.ldy = p.ldy;
    g.y_batch = p.y_batch;
    g.alpha = p.alpha;
    g.beta = p.beta;
    g.part = p.part;
    g.causal = p.causal;
    g.c_grp = p.c_grp > 0 ? p.c_grp : 1;
    g.c_start = p.c_start;
    g.c_seg = p.c_seg;
    g.c_seglen = p.c_seglen;
    g.err = p.err;
    CUtensorMap ma, mb;
    const long long arows = p.batch > 1 ? (long long)p.batch * p.a_batch_rows : p.M;
    const long long brows = p.batch > 1 ? (long long)p.batch * p.b_batch_rows : p.N;
    if ((e = make_map(&ma, A, arows, p.K, lda, BM)) != cudaSuccess) return e;
    if ((e = make_map(&mb, B, brows, p.K, ldb, BN)) != cudaSuccess) return e;
    const long long tiles = (long long)g.batch * g.mt * g.nt * g.ks;
    const int grid = (int)(tiles < g_sm_count[dev] ? tiles : g_sm_count[dev]);
    fl_tc_gemm_kernel<BN><<<grid, kThreads, C::SMEM, st>>>(ma, mb, g);
    e = cudaGetLastError();
    if (e != cudaSuccess || g.ks == 1) return e;
    const long long count = (long long)g.batch * g.N * g.M;
    const long long blocks = std::min<long long>((count + 255) / 256, (long long)g_sm_count[dev] * 8);
    split_reduce_kernel<<<(unsigned)blocks, 256, 0, st>>>(g.part, g.ks, g.batch, g.N, g.M, g.Y, g.ldy, g.y_batch,
                                                           g.alpha, g.beta);
    return cudaGetLastError();
}

} // namespace

size_t fl_tc_gemm_smem_bytes(int bn)
{
    return bn >= 256 ? Cfg<256>::SMEM : (bn >= 128 ? Cfg<128>::SMEM : Cfg<64>::SMEM);
}

cudaError_t fl_tc_gemm(const __half* A, long long lda, const __half* B, long long ldb, const FlTcGemm& p,
                       cudaStream_t st)
{
    if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.batch <= 0 || !p.Y) return cudaErrorInvalidValue;
    if (p.batch > 1 && (p.a_batch_rows < p.M || p.b_batch_rows < p.N)) return cudaErrorInvalidValue;
    if (p.ksplit > 1 && (!p.part || p.causal)) return cudaErrorInvalidValue;
    if (p.causal == 2 && (p.c_seglen % BK || (long long)p.c_seg * p.c_seglen != p.K)) return cudaErrorInvalidValue;
    /* the token tile: as wide as the token count needs, at most 256 */
    if (p.N > 128) return launch<256>(A, lda, B, ldb, p, st);
    if (p.N > 64) return launch<128>(A, lda, B, ldb, p, st);
    return launch<64>(A, lda, B, ldb, p, st);
}
