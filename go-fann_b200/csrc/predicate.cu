// predicate.cu — predicate pass bitmaps of candidate rows.
//
// The reference's traversal can evaluate the DNF predicate of one
// expansion's candidates with one lane per candidate and a warp ballot, so
// that the pass bits keep candidate order for the serial heap updates
// (prepare_candidate_pass_masks, src/predicates/gpu_predicate_parallel.cuh:
// 21-42).  The same bitmap over a flat candidate list: candidate i is local
// row cand_rows[i] of route cand_route[i]'s graph group; lane i % 32 of a
// warp decides it, and the warp's ballot is word i / 32 of the output.
#include "common.cuh"

namespace gofann {
namespace {

__global__ void pass_mask_kernel(gofann_graph g, AttrView at, gofann_routes r, const uint32_t* __restrict__ cand_route,
                                 const uint32_t* __restrict__ cand_rows, uint32_t n, uint32_t* __restrict__ out,
                                 int32_t* status)
{
    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (blockDim.x / 32);
    for (uint64_t w = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; w * 32 < n;
         w += warps) {
        const uint64_t i = w * 32 + lane;
        bool pass = false;
        if (i < n) {
            const uint32_t route = cand_route[i];
            bool ok = route < r.n_routes;
            const uint32_t grp = ok ? r.group_id[route] : 0u;
            ok = ok && grp < g.group_count;
            const uint64_t grow = ok ? static_cast<uint64_t>(g.label_offset[grp]) + cand_rows[i] : 0u;
            ok = ok && grow < g.total_rows;
            if (!ok) {
                if (status) atomicExch(status, GOFANN_ERR_INVALID);
            } else {
                const uint32_t sample = g.row_to_sample[grow];
                pass = pred_enabled(r, route) ? pred_matches(r, at, route, sample) : true;
            }
        }
        const unsigned m = __ballot_sync(kFull, pass);
        if (lane == 0) out[w] = m;
    }
}

}  // namespace
}  // namespace gofann

using namespace gofann;

extern "C" {

int gofann_predicate_pass_masks(const gofann_graph* graph, const gofann_attrs* attrs, const gofann_routes* routes,
                                const uint32_t* cand_route, const uint32_t* cand_rows, uint32_t n_candidates,
                                uint32_t* out_masks, int32_t* status, void* stream)
{
    if (!graph || !attrs || !routes || !cand_route || !cand_rows || !out_masks)
        return fail(GOFANN_ERR_INVALID, "predicate_pass_masks: null argument");
    if (!graph->row_to_sample || !graph->label_offset || !routes->group_id)
        return fail(GOFANN_ERR_INVALID, "predicate_pass_masks: row_to_sample, label_offset and group_id required");
    if (routes->pred_offsets && (!attrs->label_indptr || !routes->clauses || !routes->pred_handles))
        return fail(GOFANN_ERR_INVALID, "predicate_pass_masks: predicate arrays missing");
    if (n_candidates == 0) return GOFANN_OK;
    const AttrView at = make_attr_view(attrs);
    const int threads = 256;
    const uint64_t want = (static_cast<uint64_t>(n_candidates) + threads - 1) / threads;
    const int sms = sm_count() > 0 ? sm_count() : 148;
    const unsigned blocks = static_cast<unsigned>(want < static_cast<uint64_t>(sms) * 16 ? want : sms * 16);
    pass_mask_kernel<<<blocks, threads, 0, as_stream(stream)>>>(*graph, at, *routes, cand_route, cand_rows,
                                                               n_candidates, out_masks, status);
    GOFANN_CHECK_LAUNCH("pass_mask_kernel");
    return GOFANN_OK;
}

}  // extern "C"
