// beam_variants_u8.cu — the integer-codebook PQ traversal variants (GOFANN_PQ_U8)
// (kept in a file of their own so that the variants compile in parallel).
#include "beam_kernel.cuh"

namespace gofann {
namespace beam {

template <bool kExt>
KernelFn pick_u8_ext(bool bias, bool w4, bool small_m)
{
    if (bias) {
        if (w4) return small_m ? beam_search_kernel<0, true, GOFANN_PQ_U8, 4, 64, kExt>
                               : beam_search_kernel<0, true, GOFANN_PQ_U8, 4, 128, kExt>;
        return small_m ? beam_search_kernel<0, true, GOFANN_PQ_U8, 0, 64, kExt>
                       : beam_search_kernel<0, true, GOFANN_PQ_U8, 0, 128, kExt>;
    }
    if (w4) return small_m ? beam_search_kernel<0, false, GOFANN_PQ_U8, 4, 64, kExt>
                           : beam_search_kernel<0, false, GOFANN_PQ_U8, 4, 128, kExt>;
    return small_m ? beam_search_kernel<0, false, GOFANN_PQ_U8, 0, 64, kExt>
                   : beam_search_kernel<0, false, GOFANN_PQ_U8, 0, 128, kExt>;
}

KernelFn pick_u8(bool bias, bool w4, bool small_m, bool ext)
{
    return ext ? pick_u8_ext<true>(bias, w4, small_m) : pick_u8_ext<false>(bias, w4, small_m);
}

}  // namespace beam
}  // namespace gofann
