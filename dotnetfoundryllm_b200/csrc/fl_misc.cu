/*
 * fl_misc.cu — bit-exact dequantization (Dequantizer.cs, the fl_dequant entry
 * point) and top-k over the device logits (fl_topk).
 */
#include <float.h>
#include <math.h>

#include "fl_decode.h"
#include "fl_dequant.cuh"
#include "fl_device.cuh"
#include "fl_kernels.h"
#include "../../include/foundry_cuda.h"

namespace {

__global__ void fl_dequant_kernel(int type, const uint8_t* __restrict__ src, int64_t n, float* __restrict__ dst)
{
    for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < n; f += (int64_t)gridDim.x * blockDim.x)
        dst[f] = fl_dequant_elem(type, src, f);
}

/* ── top-k ──────────────────────────────────────────────────────────────
 * TopKSampler.ApplyTopK (TopKSampler.cs:42-71) keeps every logit >= the k-th
 * largest; the selection here returns the k winners in (value descending,
 * index ascending) order:
 *  1. radix select of the k-th largest on order-preserving keys (4 passes of
 *     8 bits), which also yields how many keys equal to it are needed;
 *  2. the keys strictly above it (fewer than k) are gathered and sorted as
 *     (key, ~index) pairs: a bitonic sort in shared memory, or for more than
 *     SORT_CAP of them sorted chunks merged by binary-search ranks;
 *  3. the tied keys are taken in index order by a block-wide ordered scan,
 *     straight into their final positions.
 * Every step is O(n) or O(k log k): all-equal logits cost one scan. */
constexpr int TOPK_THREADS = 1024;
constexpr int SORT_CAP = 4096;

/* -0 and +0 compare equal (as the reference's float compares do), so -0 is
 * keyed as +0; ties between them then go by index. */
__device__ __forceinline__ uint32_t order_key(float f)
{
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/* Descending bitonic sort of a[0..N) (N a power of two, <= SORT_CAP). */
__device__ void bitonic_desc(uint64_t* a, int N)
{
    for (int size = 2; size <= N; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < N / 2; i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
                const uint64_t A = a[lo], B = a[hi];
                if ((A < B) == ((lo & size) == 0)) {
                    a[lo] = B;
                    a[hi] = A;
                }
            }
        }
    __syncthreads();
}

/* Elements of a descending array a[0..len) greater than v. */
__device__ __forceinline__ int count_greater(const uint64_t* a, int len, uint64_t v)
{
    int lo = 0, hi = len;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (a[mid] > v) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

__device__ __forceinline__ void emit(const float* x, uint64_t c, int rank, int* ids, float* vals)
{
    const int idx = (int)(0xFFFFFFFFu - (uint32_t)c);
    ids[rank] = idx;
    vals[rank] = x[idx];
}

__global__ void __launch_bounds__(TOPK_THREADS) fl_topk_kernel(const float* __restrict__ x, int n, int k,
                                                               int* __restrict__ ids, float* __restrict__ vals,
                                                               uint64_t* __restrict__ cand, int cand_cap)
{
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_k, s_cnt, s_base;
    __shared__ int s_warp[TOPK_THREADS / 32];
    __shared__ uint64_t srt[SORT_CAP];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        s_prefix = 0;
        s_mask = 0;
        s_k = k;
        s_cnt = 0;
        s_base = 0;
    }
    __syncthreads();
    /* 1. radix select */
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int i = tid; i < n; i += blockDim.x) {
            const uint32_t key = order_key(x[i]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFF], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            int need = s_k;
            int b = 255;
            for (; b > 0; b--) {
                if ((int)hist[b] >= need) break;
                need -= (int)hist[b];
            }
            s_k = need;
            s_prefix = prefix | ((uint32_t)b << shift);
            s_mask = mask | (0xFFu << shift);
        }
        __syncthreads();
    }
    const uint32_t thr = s_prefix; /* key of the k-th largest */
    const int need = s_k;          /* keys equal to thr among the k */
    const int above = k - need;    /* keys strictly above thr */

    /* 2a. gather the keys above the threshold (unordered) */
    for (int i = tid; i < n; i += blockDim.x) {
        const uint32_t key = order_key(x[i]);
        if (key > thr) {
            const int p = atomicAdd(&s_cnt, 1);
            if (p < cand_cap) cand[p] = ((uint64_t)key << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)i);
        }
    }
    /* 3. the first `need` tied keys in index order, at ranks above.. */
    for (int c0 = 0; c0 < n; c0 += blockDim.x) {
        __syncthreads();
        const int base = s_base;
        if (base >= need) break; /* uniform: every thread read the same s_base */
        const int i = c0 + tid;
        const bool tie = i < n && order_key(x[i]) == thr;
        const uint32_t bal = __ballot_sync(0xffffffffu, tie);
        if (lane == 0) s_warp[warp] = __popc(bal);
        __syncthreads();
        int before = 0, total = 0;
        for (int w = 0; w < TOPK_THREADS / 32; w++) {
            const int cw = s_warp[w];
            if (w < warp) before += cw;
            total += cw;
        }
        const int r = base + before + __popc(bal & ((1u << lane) - 1u));
        if (tie && r < need) {
            ids[above + r] = i;
            vals[above + r] = x[i];
        }
        __syncthreads();
        if (tid == 0) s_base = base + total;
    }
    __syncthreads();
    /* 2b. rank the keys above */
    const int m = min(above, cand_cap);
    if (m <= SORT_CAP) {
        int N = 1;
        while (N < m) N <<= 1;
        for (int i = tid; i < N; i += blockDim.x) srt[i] = i < m ? cand[i] : 0ull;
        bitonic_desc(srt, N);
        for (int i = tid; i < m; i += blockDim.x) emit(x, srt[i], i, ids, vals);
        return;
    }
    /* more than SORT_CAP: sort chunks of SORT_CAP in place, then merge ranks */
    const int nchunk = (m + SORT_CAP - 1) / SORT_CAP;
    for (int c = 0; c < nchunk; c++) {
        const int lo = c * SORT_CAP, len = min(SORT_CAP, m - lo);
        __syncthreads();
        for (int i = tid; i < SORT_CAP; i += blockDim.x) srt[i] = i < len ? cand[lo + i] : 0ull;
        bitonic_desc(srt, SORT_CAP);
        for (int i = tid; i < len; i += blockDim.x) cand[lo + i] = srt[i];
    }
    __syncthreads();
    for (int e = tid; e < m; e += blockDim.x) {
        const int c = e / SORT_CAP;
        const uint64_t v = cand[e];
        int rank = e - c * SORT_CAP;
        for (int o = 0; o < nchunk; o++)
            if (o != c) rank += count_greater(cand + (size_t)o * SORT_CAP, min(SORT_CAP, m - o * SORT_CAP), v);
        emit(x, v, rank, ids, vals);
    }
}

} // namespace

cudaError_t fl_launch_dequant(int32_t type, const uint8_t* src, int64_t n, float* dst, cudaStream_t st)
{
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    if (blocks < 1) blocks = 1;
    fl_dequant_kernel<<<(unsigned)blocks, 256, 0, st>>>(type, src, n, dst);
    return cudaGetLastError();
}

size_t fl_topk_scratch_bytes(int32_t n, int32_t k)
{
    (void)k;
    return (size_t)n * 8;
}

cudaError_t fl_launch_topk(const float* logits, int32_t n, int32_t k, int32_t* ids, float* vals, uint8_t* scratch,
                           size_t scratch_bytes, cudaStream_t st)
{
    const int cap = (int)(scratch_bytes / 8);
    fl_topk_kernel<<<1, TOPK_THREADS, 0, st>>>(logits, n, k, ids, vals, reinterpret_cast<uint64_t*>(scratch), cap);
    return cudaGetLastError();
}

/* Scratch of fl_topk_device: candidate keys and indices for n <= FL_TOPK_DEVICE_MAX_N. */
static __device__ __align__(256) uint8_t g_topk_device_scratch[(size_t)FL_TOPK_DEVICE_MAX_N * 8];

cudaError_t fl_launch_topk_static(const float* logits, int32_t n, int32_t k, int32_t* ids, float* vals,
                                  cudaStream_t st)
{
    /* The array's address on the current device, looked up on every call:
     * the lookup allocates nothing, and an address kept from an earlier call
     * would dangle after a cudaDeviceReset reloads the module.  Host code may
     * not pass the symbol itself: in host code it names a host-side stand-in. */
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_topk_device_scratch);
    if (e != cudaSuccess) return e;
    return fl_launch_topk(logits, n, k, ids, vals, static_cast<uint8_t*>(p), (size_t)FL_TOPK_DEVICE_MAX_N * 8, st);
}
