// beam_variants_direct.cu — the PQ traversal variants that evaluate table entries from the query and codebook (GOFANN_PQ_DIRECT)
// (kept in a file of their own so that the variants compile in parallel).
#include "beam_kernel.cuh"

namespace gofann {
namespace beam {

template <bool kExt>
KernelFn pick_direct_ext(bool bias, bool w4, bool small_m)
{
    if (bias) {
        if (w4) return small_m ? beam_search_kernel<0, true, GOFANN_PQ_DIRECT, 4, 64, kExt>
                               : beam_search_kernel<0, true, GOFANN_PQ_DIRECT, 4, 128, kExt>;
        return small_m ? beam_search_kernel<0, true, GOFANN_PQ_DIRECT, 0, 64, kExt>
                       : beam_search_kernel<0, true, GOFANN_PQ_DIRECT, 0, 128, kExt>;
    }
    if (w4) return small_m ? beam_search_kernel<0, false, GOFANN_PQ_DIRECT, 4, 64, kExt>
                           : beam_search_kernel<0, false, GOFANN_PQ_DIRECT, 4, 128, kExt>;
    return small_m ? beam_search_kernel<0, false, GOFANN_PQ_DIRECT, 0, 64, kExt>
                   : beam_search_kernel<0, false, GOFANN_PQ_DIRECT, 0, 128, kExt>;
}

KernelFn pick_direct(bool bias, bool w4, bool small_m, bool ext)
{
    return ext ? pick_direct_ext<true>(bias, w4, small_m) : pick_direct_ext<false>(bias, w4, small_m);
}

}  // namespace beam
}  // namespace gofann
