/* fl_token_hd128.cu — token-kernel instances for head_dim 128 (one per largest
 * query-head group, so each carries only its own attention variant). */
#include "fl_token.cuh"

const void* fl_token_kernel_hd128(int gmax)
{
    switch (gmax) {
    case 1: return fltk::kernel_ptr<128, 1>();
    case 2: return fltk::kernel_ptr<128, 2>();
    case 4: return fltk::kernel_ptr<128, 4>();
    case 8: return fltk::kernel_ptr<128, 8>();
    default: return nullptr;
    }
}
