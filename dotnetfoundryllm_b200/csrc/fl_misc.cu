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
 * Radix select of the k-th largest on order-preserving keys, then the
 * (value desc, index asc) order of the k winners. */
__device__ __forceinline__ uint32_t order_key(float f)
{
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void fl_topk_kernel(const float* __restrict__ x, int n, int k, int* __restrict__ ids,
                               float* __restrict__ vals, uint32_t* __restrict__ cand_key, int* __restrict__ cand_idx,
                               int cand_cap)
{
    /* single CTA of 1024 threads */
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_k, s_cnt;
    if (threadIdx.x == 0) {
        s_prefix = 0;
        s_mask = 0;
        s_k = k;
        s_cnt = 0;
    }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            uint32_t key = order_key(x[i]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFF], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
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
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        uint32_t key = order_key(x[i]);
        if (key >= thr) {
            int p = atomicAdd(&s_cnt, 1);
            if (p < cand_cap) {
                cand_key[p] = key;
                cand_idx[p] = i;
            }
        }
    }
    __syncthreads();
    const int m = min(s_cnt, cand_cap);
    /* rank each candidate: larger key first, then lower index */
    for (int c = threadIdx.x; c < m; c += blockDim.x) {
        uint32_t kc = cand_key[c];
        int ic = cand_idx[c];
        int rank = 0;
        for (int o = 0; o < m; o++) {
            uint32_t ko = cand_key[o];
            int io = cand_idx[o];
            rank += (ko > kc) || (ko == kc && io < ic);
        }
        if (rank < k) {
            ids[rank] = ic;
            vals[rank] = x[ic];
        }
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
    int cap = (int)(scratch_bytes / 8);
    uint32_t* ck = reinterpret_cast<uint32_t*>(scratch);
    int* ci = reinterpret_cast<int*>(scratch + (size_t)cap * 4);
    fl_topk_kernel<<<1, 1024, 0, st>>>(logits, n, k, ids, vals, ck, ci, cap);
    return cudaGetLastError();
}

/* Scratch of fl_topk_device: candidate keys and indices for n <= FL_TOPK_DEVICE_MAX_N. */
static __device__ __align__(256) uint8_t g_topk_device_scratch[(size_t)FL_TOPK_DEVICE_MAX_N * 8];

cudaError_t fl_launch_topk_static(const float* logits, int32_t n, int32_t k, int32_t* ids, float* vals,
                                  cudaStream_t st)
{
    /* address of the scratch per device, looked up on the first call */
    static void* addr[FL_MAX_DEVICES] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= FL_MAX_DEVICES) return cudaErrorInvalidDevice;
    void* p = __atomic_load_n(&addr[dev], __ATOMIC_ACQUIRE);
    if (!p) {
        e = cudaGetSymbolAddress(&p, g_topk_device_scratch);
        if (e != cudaSuccess) return e;
        __atomic_store_n(&addr[dev], p, __ATOMIC_RELEASE);
    }
    return fl_launch_topk(logits, n, k, ids, vals, static_cast<uint8_t*>(p), (size_t)FL_TOPK_DEVICE_MAX_N * 8, st);
}
