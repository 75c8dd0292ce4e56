/*
 * fl_token.cu — host side of the persistent token kernel (fl_token.cuh):
 * instance selection, shared-memory sizing, configuration and launch.
 */
#include "fl_token.cuh"

const void* fl_token_kernel_hd64(int gmax);
const void* fl_token_kernel_hd128(int gmax);
const void* fl_token_kernel_hd256(int gmax);

const void* fl_token_kernel_ptr(int head_dim, int group)
{
    int gmax = 0;
    for (int g = 1; g <= 8 && !gmax; g <<= 1)
        if (group <= g) gmax = g;
    if (group < 1 || !gmax) return nullptr;
    switch (head_dim) {
    case 64: return fl_token_kernel_hd64(gmax);
    case 128: return fl_token_kernel_hd128(gmax);
    case 256: return fl_token_kernel_hd256(gmax);
    default: return nullptr;
    }
}

size_t fl_token_smem_bytes(int n_slots, int slot_bytes, size_t scratch_bytes, int n_feed)
{
    return fltk::tk_layout(n_slots, slot_bytes, scratch_bytes, n_feed).total;
}

cudaError_t fl_token_configure(const void* kernel, int* max_dyn_smem)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return e;
    const int avail = optin - (int)fa.sharedSizeBytes;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, avail);
    if (e == cudaSuccess && max_dyn_smem) *max_dyn_smem = avail;
    return e;
}

cudaError_t fl_launch_token(const void* kernel, const FlTokenArgs& ta, int grid, size_t smem, cudaStream_t st)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(fltk::NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {const_cast<FlTokenArgs*>(&ta)};
    return cudaLaunchKernelExC(&cfg, kernel, args);
}
