/* fl_token_hd256.cu — token-kernel instances for head_dim 256 (one per largest
 * query-head group, so each carries only its own attention variant). */
#include "fl_token.cuh"

const void* fl_token_kernel_hd256(int gmax)
{
    switch (gmax) {
    case 1: return fltk::kernel_ptr<256, 1>();
    case 2: return fltk::kernel_ptr<256, 2>();
    case 4: return fltk::kernel_ptr<256, 4>();
    default: return nullptr;
    }
}
