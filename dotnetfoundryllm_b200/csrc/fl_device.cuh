/*
 * fl_device.cuh — sm_100a device helpers: mbarriers, bulk async copies,
 * programmatic dependent launch, the int8 tensor-core MMA, bounded waits.
 */
#ifndef FL_DEVICE_CUH
#define FL_DEVICE_CUH

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define FL_DEV_ERR_TIMEOUT 1
#define FL_DEV_ERR_TOKEN 2
#define FL_DEV_ERR_RANGE 3 /* a prompt-path operand outside the fp16 range of its tensor-core GEMM */

__device__ __forceinline__ uint32_t fl_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void fl_mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(fl_smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fl_fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void fl_mbar_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fl_smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool fl_mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(fl_smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t fl_globaltimer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

/* An error already recorded by a bounded wait of this launch (or an earlier
 * phase): later waits on other CTAs or ranks return at once, so a launch that
 * lost a peer ends after one wait limit instead of one per exchange. */
__device__ __forceinline__ bool fl_err_set(const int* err) { return err && *(volatile const int*)err != 0; }

/* Bounded wait on an mbarrier phase: gives up after ~2 s (or 2^26 polls),
 * records FL_DEV_ERR_TIMEOUT in *err and returns false.  Never traps. */
/* Non-blocking test of a phase's completion. */
__device__ __forceinline__ bool fl_mbar_test(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(fl_smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void fl_mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(fl_smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool fl_mbar_wait(uint64_t* bar, uint32_t parity, int* err)
{
    if (fl_mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = fl_globaltimer();
    for (uint32_t it = 0; it < (1u << 26); ++it) {
        if (fl_mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0 && fl_globaltimer() - t0 > 2000000000ull) break;
    }
    if (err) atomicExch(err, FL_DEV_ERR_TIMEOUT);
    return false;
}

/* 1-D bulk copy global → shared, completion counted on an mbarrier.  Both
 * addresses 16-byte aligned, size a multiple of 16.  No multicast. */
__device__ __forceinline__ void fl_bulk_g2s(void* sdst, const void* gsrc, uint32_t bytes, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            fl_smem_u32(sdst)),
        "l"(gsrc), "r"(bytes), "r"(fl_smem_u32(bar))
        : "memory");
}

/* System-scope release store / acquire load: flags between GPUs (peer memory
 * mapped over NVLink). */
__device__ __forceinline__ void fl_st_release_sys(int* p, int v)
{
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int fl_ld_acquire_sys(const int* p)
{
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

/* Coherent (system-scope) load of a value another GPU may have written. */
__device__ __forceinline__ float fl_ld_relaxed_sys(const float* p)
{
    float v;
    asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

/* Two 8-byte words, each read atomically, through L2 every time (polling
 * words another CTA or GPU writes with single 8-byte stores). */
__device__ __forceinline__ ulonglong2 fl_ld_volatile_u64x2(const ulonglong2* p)
{
    ulonglong2 v;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}

/* Asks L2 to fetch [p, p + bytes) (16-byte aligned, size a multiple of 16). */
__device__ __forceinline__ void fl_prefetch_l2(const void* p, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

/* Orders this thread's earlier generic-proxy shared accesses before later
 * async-proxy (bulk copy) writes to the same shared memory. */
__device__ __forceinline__ void fl_fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

/* Programmatic dependent launch. */
__device__ __forceinline__ void fl_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void fl_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

/* D(16x8, s32) = A(16x32) * B(32x8), A u8 or s8, B s8, C = 0. */
template <bool SIGNED_A>
__device__ __forceinline__ void fl_mma_i8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    if constexpr (SIGNED_A) {
        asm(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%10,%10,%10};\n"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
    } else {
        asm(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%10,%10,%10};\n"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
    }
}

__device__ __forceinline__ float fl_warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float fl_warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

/* Block reduction of two values (sum, max) over blockDim.x threads. */
__device__ __forceinline__ void fl_block_sum_max(float& s, float& m, float* scratch /* 2*32 floats */)
{
    s = fl_warp_sum(s);
    m = fl_warp_max(m);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (lane == 0) {
        scratch[warp] = s;
        scratch[32 + warp] = m;
    }
    __syncthreads();
    float ts = 0.0f, tm = 0.0f;
    for (int w = 0; w < nw; w++) {
        ts += scratch[w];
        tm = fmaxf(tm, scratch[32 + w]);
    }
    s = ts;
    m = tm;
}

/* TensorPrimitives.IndexOfMax order: NaN first, then larger value, +0 over
 * -0, then the lower index. */
__device__ __forceinline__ bool fl_argmax_better(float a, int ia, float b, int ib)
{
    bool na = a != a, nb = b != b;
    if (na || nb) {
        if (na && nb) return ia < ib;
        return na;
    }
    if (a > b) return true;
    if (a < b) return false;
    if (a == 0.0f) {
        bool sa = signbit(a), sb = signbit(b);
        if (sa != sb) return !sa;
    }
    return ia < ib;
}

#endif
