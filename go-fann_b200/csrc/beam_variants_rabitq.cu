// beam_variants_rabitq.cu — the 1-bit RaBitQ traversal variants
// (kept in a file of their own so that the variants compile in parallel).
#include "beam_kernel.cuh"

namespace gofann {
namespace beam {

KernelFn pick_rabitq(bool bias, bool ext)
{
    if (ext) return bias ? beam_search_kernel<1, true, 0, 0, 64, true> : beam_search_kernel<1, false, 0, 0, 64, true>;
    return bias ? beam_search_kernel<1, true, 0, 0, 64, false> : beam_search_kernel<1, false, 0, 0, 64, false>;
}

}  // namespace beam
}  // namespace gofann
