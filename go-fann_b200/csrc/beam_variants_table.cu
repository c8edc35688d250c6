// beam_variants_table.cu — the PQ traversal variants that read a per-query lookup table (GOFANN_PQ_LUT_GLOBAL / _SHARED)
// (kept in a file of their own so that the variants compile in parallel).
#include "beam_kernel.cuh"

namespace gofann {
namespace beam {

template <bool kExt>
KernelFn pick_table_ext(bool shared, bool bias, bool small_m)
{
    if (shared) {
        if (bias) return small_m ? beam_search_kernel<0, true, GOFANN_PQ_LUT_SHARED, 0, 64, kExt>
                                 : beam_search_kernel<0, true, GOFANN_PQ_LUT_SHARED, 0, 128, kExt>;
        return small_m ? beam_search_kernel<0, false, GOFANN_PQ_LUT_SHARED, 0, 64, kExt>
                       : beam_search_kernel<0, false, GOFANN_PQ_LUT_SHARED, 0, 128, kExt>;
    }
    if (bias) return small_m ? beam_search_kernel<0, true, GOFANN_PQ_LUT_GLOBAL, 0, 64, kExt>
                             : beam_search_kernel<0, true, GOFANN_PQ_LUT_GLOBAL, 0, 128, kExt>;
    return small_m ? beam_search_kernel<0, false, GOFANN_PQ_LUT_GLOBAL, 0, 64, kExt>
                   : beam_search_kernel<0, false, GOFANN_PQ_LUT_GLOBAL, 0, 128, kExt>;
}

KernelFn pick_table(bool shared, bool bias, bool small_m, bool ext)
{
    return ext ? pick_table_ext<true>(shared, bias, small_m) : pick_table_ext<false>(shared, bias, small_m);
}

}  // namespace beam
}  // namespace gofann
