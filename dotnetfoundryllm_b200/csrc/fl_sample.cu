/*
 * fl_sample.cu — the decode loop's sampling step on the device (fl_sample).
 *
 * Reference, in the order LlamaLanguageModel.GenerateAsync applies it
 * (src/DotNetFoundryLLM.Inference/LlamaLanguageModel.cs:183-216):
 *  1. ApplyRepetitionPenalty (LlamaLanguageModel.cs:357-373): for every
 *     occurrence of a token in the generated list, a positive logit is
 *     divided by the penalty and any other multiplied by it.  Occurrences of
 *     one id are applied in sequence, so the host passes (id, count) pairs and
 *     the kernel repeats the operation `count` times: the same roundings.
 *  2. SamplerPipeline.Sample (src/DotNetFoundryLLM.Sampling/SamplerPipeline.cs:58-89):
 *     temperature 0 → ArgMax; else logits * (1/T); TopKSampler.ApplyTopK
 *     (values below the k-th largest → -inf, ties kept); Softmax; TopPSampler.
 *     ApplyTopP (keep tokens by descending probability until the running sum
 *     reaches p, zero the rest, renormalize); TemperatureSampler.
 *     SampleFromProbabilities (the first index whose running sum in index
 *     order exceeds the uniform draw u).
 *
 * The draw u is the host's (XoshiroRandom.NextFloat of the request's
 * generator), so a seeded request draws the same numbers as the reference.
 * The final running sum is formed exactly as the reference does (sequential
 * float additions in index order); the softmax sum and the top-p nucleus mass
 * are reduced in a fixed order of our own (the reference's TensorPrimitives.Sum
 * order is ISA-dependent), so tokens can differ only where u lies within a
 * rounding of a CDF boundary.
 */
#include <cuda_runtime.h>
#include <stdint.h>

#include "fl_device.cuh"
#include "fl_kernels.h"

namespace {

constexpr int ST = 1024; /* threads of the single-CTA finishing kernel */

__global__ void samp_penalty_kernel(float* __restrict__ w, const int2* __restrict__ pairs, int n_pairs, float pen)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_pairs) return;
    const int2 pc = pairs[i];
    float x = w[pc.x];
    for (int c = 0; c < pc.y; c++) x = x > 0.0f ? __fdiv_rn(x, pen) : __fmul_rn(x, pen);
    w[pc.x] = x;
}

__global__ void samp_scale_kernel(float* __restrict__ w, int n, float inv)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) w[i] = __fmul_rn(w[i], inv);
}

/* ApplyTopK after the radix select: vals[k-1] is the k-th largest value. */
__global__ void samp_topk_mask_kernel(float* __restrict__ w, int n, const float* __restrict__ vals, int k)
{
    const float thr = vals[k - 1];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        if (w[i] < thr) w[i] = -INFINITY;
}

/* Block-wide reductions of the finishing kernel (fixed order: a shuffle tree
 * per warp, then warp 0 over the warps). */
__device__ float block_sum(float v, float* red)
{
    v = fl_warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < ST / 32 ? red[lane] : 0.0f;
        t = fl_warp_sum(t);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

/* Probability mass in 2^-40 units: integer sums are exact and order-free. */
__device__ __forceinline__ unsigned long long mass_of(float p)
{
    return (unsigned long long)((double)p * 1099511627776.0);
}

/* Greedy, or softmax → top-p → sampling, on w[0..n) in one CTA. */
__global__ void __launch_bounds__(ST, 1)
    samp_finish_kernel(float* __restrict__ w, int n, int greedy, float top_p, float u, int* __restrict__ token)
{
    __shared__ float redf[33];
    __shared__ unsigned long long redu[33];
    __shared__ unsigned long long hist[256];
    __shared__ int s_int[4];
    const int tid = threadIdx.x;

    if (greedy) {
        /* TensorPrimitives.IndexOfMax: the first maximum (a NaN wins at once) */
        float bv = 0.0f;
        int bi = 0x7fffffff;
        for (int i = tid; i < n; i += ST) {
            const float v = w[i];
            if (bi == 0x7fffffff || fl_argmax_better(v, i, bv, bi)) {
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
        if ((tid & 31) == 0) {
            redf[tid >> 5] = bv;
            redu[tid >> 5] = (unsigned long long)(unsigned)bi;
        }
        __syncthreads();
        if (tid == 0) {
            float v = redf[0];
            int b = (int)redu[0];
            for (int q = 1; q < ST / 32; q++) {
                const int oi = (int)redu[q];
                if (oi != 0x7fffffff && (b == 0x7fffffff || fl_argmax_better(redf[q], oi, v, b))) {
                    v = redf[q];
                    b = oi;
                }
            }
            *token = b;
        }
        return;
    }

    /* Softmax (TensorOperations.cs:23-39): max, x + (-max), exp, sum, divide */
    /* TensorPrimitives.Max: NaN if any value is NaN */
    float mx = -INFINITY;
    int nan = 0;
    for (int i = tid; i < n; i += ST) {
        const float v = w[i];
        nan |= isnan(v);
        mx = fmaxf(mx, v);
    }
    nan = __syncthreads_or(nan);
    mx = fl_warp_max(mx);
    if ((tid & 31) == 0) redf[tid >> 5] = mx;
    __syncthreads();
    if (tid == 0) {
        float t = redf[0];
        for (int q = 1; q < ST / 32; q++) t = fmaxf(t, redf[q]);
        redf[32] = t;
    }
    __syncthreads();
    mx = nan ? __int_as_float(0x7fc00000) : redf[32];
    __syncthreads();
    float part = 0.0f;
    for (int i = tid; i < n; i += ST) {
        const float e = expf(__fadd_rn(w[i], -mx));
        w[i] = e;
        part = __fadd_rn(part, e);
    }
    const float sum = block_sum(part, redf);
    if (sum != 0.0f)
        for (int i = tid; i < n; i += ST) w[i] = __fdiv_rn(w[i], sum);
    __syncthreads();

    /* TopPSampler.ApplyTopP (TopPSampler.cs:60-110) */
    if (top_p < 1.0f && !nan) {
        const unsigned long long P = mass_of(top_p);
        unsigned long long above = 0; /* mass of the values above the current prefix range */
        uint32_t prefix = 0;
        int keep_all = 0;
        for (int level = 0; level < 4 && !keep_all; level++) {
            const int shift = 24 - 8 * level;
            const uint32_t hmask = level == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
            for (int b = tid; b < 256; b += ST) hist[b] = 0ull;
            __syncthreads();
            for (int i = tid; i < n; i += ST) {
                const uint32_t bits = __float_as_uint(w[i]);
                if ((bits & hmask) == prefix) atomicAdd(&hist[(bits >> shift) & 0xFFu], mass_of(w[i]));
            }
            __syncthreads();
            if (tid == 0) {
                unsigned long long acc = 0;
                int found = -1;
                for (int b = 255; b >= 0; b--) {
                    if (above + acc + hist[b] >= P) {
                        found = b;
                        break;
                    }
                    acc += hist[b];
                }
                if (found < 0) {
                    s_int[0] = 1; /* the nucleus is never reached: nothing is removed */
                } else {
                    s_int[0] = 0;
                    above += acc;
                    prefix |= (uint32_t)found << shift;
                }
                redu[0] = above;
                s_int[1] = (int)prefix;
            }
            __syncthreads();
            keep_all = s_int[0];
            above = redu[0];
            prefix = (uint32_t)s_int[1];
            __syncthreads();
        }
        if (!keep_all && prefix != 0u) {
            /* values above the threshold stay; of the values equal to it, the
             * first m in index order, m the fewest that reach p */
            const unsigned long long mt = mass_of(__uint_as_float(prefix));
            const int chunk = (n + ST - 1) / ST, lo = tid * chunk, hi = min(n, lo + chunk);
            int ties = 0;
            for (int i = lo; i < hi; i++) ties += __float_as_uint(w[i]) == prefix;
            /* exclusive scan of the tie counts in thread (= index) order */
            int incl = ties;
            const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            __shared__ int wsum[32];
            if (lane == 31) wsum[warp] = incl;
            __syncthreads();
            if (tid == 0) {
                int acc = 0;
                for (int q = 0; q < ST / 32; q++) {
                    const int t = wsum[q];
                    wsum[q] = acc;
                    acc += t;
                }
                s_int[2] = acc;
            }
            __syncthreads();
            int rank = wsum[warp] + incl - ties;
            const int total_ties = s_int[2];
            long long m = total_ties;
            if (mt > 0) {
                const unsigned long long need = P > above ? P - above : 0ull;
                m = (long long)((need + mt - 1) / mt);
                if (m < 1) m = 1;
                if (m > total_ties) m = total_ties;
            }
            for (int i = lo; i < hi; i++) {
                const uint32_t bits = __float_as_uint(w[i]);
                if (bits < prefix) w[i] = 0.0f;
                else if (bits == prefix) {
                    if (rank >= m) w[i] = 0.0f;
                    rank++;
                }
            }
            __syncthreads();
        }
        /* renormalized whether or not anything was removed, as the reference does */
        part = 0.0f;
        for (int i = tid; i < n; i += ST) part = __fadd_rn(part, w[i]);
        const float s2 = block_sum(part, redf);
        if (s2 > 0.0f)
            for (int i = tid; i < n; i += ST) w[i] = __fdiv_rn(w[i], s2);
        __syncthreads();
    }

    /* TemperatureSampler.SampleFromProbabilities (TemperatureSampler.cs:53-70):
     * warp 0 walks w in index order, 32 values per step, adding the non-zero
     * ones in sequence exactly as the reference's loop does */
    if (tid < 32) {
        float cum = 0.0f;
        int found = -1;
        for (int base = 0; base < n && found < 0; base += 32) {
            const int i = base + tid;
            const float v = i < n ? w[i] : 0.0f;
            unsigned nz = __ballot_sync(0xffffffffu, v != 0.0f);
            while (nz) {
                const int b = __ffs(nz) - 1;
                nz &= nz - 1;
                cum = __fadd_rn(cum, __shfl_sync(0xffffffffu, v, b));
                if (u < cum) {
                    found = base + b;
                    break;
                }
            }
        }
        if (tid == 0) s_int[3] = found;
    }
    __syncthreads();
    if (s_int[3] >= 0) {
        if (tid == 0) *token = s_int[3];
        return;
    }
    /* rounding fallback: the last token with non-zero probability, else n-1 */
    int last = -1;
    for (int i = tid; i < n; i += ST)
        if (w[i] > 0.0f) last = i;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
    if ((tid & 31) == 0) redu[tid >> 5] = (unsigned long long)(long long)last;
    __syncthreads();
    if (tid == 0) {
        long long b = -1;
        for (int q = 0; q < ST / 32; q++) b = max(b, (long long)redu[q]);
        *token = b >= 0 ? (int)b : n - 1;
    }
}

} // namespace

cudaError_t fl_launch_sample_penalty(float* w, const int2* pairs, int n_pairs, float penalty, cudaStream_t st)
{
    if (n_pairs <= 0) return cudaSuccess;
    samp_penalty_kernel<<<(n_pairs + 255) / 256, 256, 0, st>>>(w, pairs, n_pairs, penalty);
    return cudaGetLastError();
}

cudaError_t fl_launch_sample_scale(float* w, int n, float inv, cudaStream_t st)
{
    samp_scale_kernel<<<148, 512, 0, st>>>(w, n, inv);
    return cudaGetLastError();
}

cudaError_t fl_launch_sample_topk_mask(float* w, int n, const float* vals, int k, cudaStream_t st)
{
    samp_topk_mask_kernel<<<148, 512, 0, st>>>(w, n, vals, k);
    return cudaGetLastError();
}

cudaError_t fl_launch_sample_finish(float* w, int n, int greedy, float top_p, float u, int* token, cudaStream_t st)
{
    samp_finish_kernel<<<1, ST, 0, st>>>(w, n, greedy, top_p, u, token);
    return cudaGetLastError();
}
