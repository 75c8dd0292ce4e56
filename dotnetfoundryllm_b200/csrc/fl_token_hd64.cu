/* fl_token_hd64.cu — token-kernel instances for head_dim 64 (one per largest
 * query-head group, so each carries only its own attention variant). */
#include "fl_token.cuh"

const void* fl_token_kernel_hd64(int gmax)
{
    switch (gmax) {
    case 1: return fltk::kernel_ptr<64, 1>();
    case 2: return fltk::kernel_ptr<64, 2>();
    case 4: return fltk::kernel_ptr<64, 4>();
    case 8: return fltk::kernel_ptr<64, 8>();
    default: return nullptr;
    }
}
