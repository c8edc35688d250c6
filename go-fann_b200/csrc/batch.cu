// batch.cu — one filtered-search batch behind a single C call.
//
// The per-stage entry points (gofann_pq_build_lut, gofann_beam_search,
// gofann_posting_scan, gofann_rerank, gofann_route_merge and the RaBitQ
// preparation) run in the reference's order on one stream, out of one
// caller-provided scratch block, so that a C or C++ host can replace the
// reference's batch driver (execute_graph_batch and its lowfreq / rerank /
// merge stages, backend_pq.cu:9740-10185, 10769, 2479-2592, 13205-13226;
// the RaBitQ batch, backend_rabitq.cu:13762-13776) with one call.  The
// scratch layout is a pure function of the batch shape, computed the same
// way by gofann_search_batch_scratch_bytes and gofann_search_batch.
#include "common.cuh"

namespace gofann {
namespace {

constexpr size_t kAlign = 256;

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Offsets of every scratch region (bytes from the scratch base).
struct BatchLayout {
    size_t lut = 0, beam = 0, beam_bytes = 0, g_ids = 0, g_d = 0, g_steps = 0, p_ids = 0, p_d = 0, r_ids = 0,
           r_d = 0, rotated = 0, q8 = 0, scale = 0, k1 = 0, gdist = 0, gemm = 0, gemm_bytes = 0, start = 0,
           total = 0;
    bool has_lut = false;  // offsets start at 0: a flag, not a zero test
};

int check_shape(const gofann_index* ix, const gofann_batch* b, const gofann_batch_params* p)
{
    if (!ix || !b || !p) return fail(GOFANN_ERR_INVALID, "search_batch: null argument");
    if (p->topk < 1 || p->topk > GOFANN_MAX_TOPK)
        return fail(GOFANN_ERR_INVALID, "search_batch: topk %d outside 1..%d", p->topk, GOFANN_MAX_TOPK);
    const uint32_t npo = b->posting_routes.n_routes;
    if (npo && (p->posting_shortlist < 1 || p->posting_shortlist > GOFANN_MAX_SHORTLIST))
        return fail(GOFANN_ERR_INVALID, "search_batch: posting shortlist %d outside 1..%d", p->posting_shortlist,
                    GOFANN_MAX_SHORTLIST);
    if (b->graph_routes.n_routes &&
        (p->search.result_width < 1 || p->search.result_width > GOFANN_MAX_RESULT_WIDTH))
        return fail(GOFANN_ERR_INVALID, "search_batch: result_width %d outside 1..%d", p->search.result_width,
                    GOFANN_MAX_RESULT_WIDTH);
    if (!b->query_route_offsets || !b->query_routes || (b->n_queries && !b->queries))
        return fail(GOFANN_ERR_INVALID, "search_batch: queries and the query -> route tables required");
    if (npo && (!b->posting_begin || !b->posting_count || !ix->posting_ids))
        return fail(GOFANN_ERR_INVALID, "search_batch: posting routes need begin, count and posting_ids");
    if (!ix->base || ix->dim == 0) return fail(GOFANN_ERR_INVALID, "search_batch: rerank store required");
    const int sc = p->search.scorer;
    if (sc == GOFANN_SCORER_RABITQ) {
        if (ix->base_dtype != GOFANN_DTYPE_F32)
            return fail(GOFANN_ERR_UNSUPPORTED, "search_batch: RaBitQ batches take f32 queries (f32 base)");
        if (!ix->rq_rotation || !ix->rq_anchors || ix->codes.padded_dim == 0 || ix->codes.num_anchors == 0)
            return fail(GOFANN_ERR_INVALID, "search_batch: RaBitQ needs rotation, anchors, padded_dim, anchors");
        if (p->rq_entries && !ix->rq_anchor_entry)
            return fail(GOFANN_ERR_INVALID, "search_batch: rq_entries needs rq_anchor_entry");
    } else if (sc != GOFANN_SCORER_PQ) {
        return fail(GOFANN_ERR_INVALID, "search_batch: unknown scorer %d", sc);
    } else if (!ix->pq_centroids) {
        return fail(GOFANN_ERR_INVALID, "search_batch: PQ needs pq_centroids");
    }
    return GOFANN_OK;
}

BatchLayout layout(const gofann_index* ix, const gofann_batch* b, const gofann_batch_params* p)
{
    BatchLayout l;
    const size_t nq = b->n_queries, ng = b->graph_routes.n_routes, npo = b->posting_routes.n_routes;
    const size_t rw = static_cast<size_t>(p->search.result_width), sl = static_cast<size_t>(p->posting_shortlist);
    const size_t k = static_cast<size_t>(p->topk);
    size_t at = 0;
    auto take = [&](size_t bytes) {
        const size_t o = at;
        at = align_up(at + bytes);
        return o;
    };
    const bool table = p->search.scorer == GOFANN_SCORER_PQ &&
                       (p->search.pq_mode == GOFANN_PQ_LUT_GLOBAL || p->search.pq_mode == GOFANN_PQ_LUT_SHARED);
    if (table) {
        l.has_lut = true;
        l.lut = take(nq * ix->codes.pq_dim * GOFANN_PQ_CENTROIDS * sizeof(float));
    }
    l.beam_bytes = gofann_beam_search_scratch_bytes(static_cast<uint32_t>(ng > 0 ? ng : 1));
    l.beam = take(l.beam_bytes);
    l.g_ids = take(ng * rw * 4);
    l.g_d = take(ng * rw * 4);
    l.g_steps = take(ng * 4);
    l.p_ids = take(npo * sl * 4);
    l.p_d = take(npo * sl * 4);
    l.r_ids = take((ng + npo) * k * 4);
    l.r_d = take((ng + npo) * k * 4);
    if (p->search.scorer == GOFANN_SCORER_RABITQ) {
        const size_t pd = ix->codes.padded_dim, na = ix->codes.num_anchors;
        l.rotated = take(nq * pd * 4);
        l.q8 = take(nq * pd);
        l.scale = take(nq * 4);
        l.k1 = take(nq * 4);
        l.gdist = take(nq * na * 4);
        const size_t g1 = gofann_rabitq_gemm_scratch_bytes(static_cast<uint32_t>(nq), ix->dim,
                                                           static_cast<uint32_t>(pd), GOFANN_GEMM_TF32X3);
        const size_t g2 = gofann_rabitq_gemm_scratch_bytes(static_cast<uint32_t>(nq), static_cast<uint32_t>(pd),
                                                           static_cast<uint32_t>(na), GOFANN_GEMM_TF32X3);
        l.gemm_bytes = g1 > g2 ? g1 : g2;
        l.gemm = take(l.gemm_bytes);
        if (p->rq_entries) l.start = take(ng * 4);
    }
    l.total = at;
    return l;
}

template <typename T>
T* at(void* base, size_t off) { return reinterpret_cast<T*>(static_cast<unsigned char*>(base) + off); }

}  // namespace
}  // namespace gofann

using namespace gofann;

extern "C" {

size_t gofann_search_batch_scratch_bytes(const gofann_index* index, const gofann_batch* batch,
                                         const gofann_batch_params* params)
{
    if (check_shape(index, batch, params) != GOFANN_OK) return 0;
    return layout(index, batch, params).total;
}

int gofann_search_batch(const gofann_index* ix, const gofann_batch* b, const gofann_batch_params* p, void* scratch,
                        size_t scratch_bytes, uint32_t* out_ids, float* out_dists, int32_t* status, void* stream)
{
    int st = check_shape(ix, b, p);
    if (st != GOFANN_OK) return st;
    if (!out_ids || !out_dists) return fail(GOFANN_ERR_INVALID, "search_batch: outputs required");
    const BatchLayout l = layout(ix, b, p);
    if (!scratch || scratch_bytes < l.total)
        return fail(GOFANN_ERR_INVALID, "search_batch: scratch of %zu bytes, %zu needed", scratch_bytes, l.total);
    if ((reinterpret_cast<uintptr_t>(scratch) & (kAlign - 1)) != 0)
        return fail(GOFANN_ERR_INVALID, "search_batch: scratch must be %zu-byte aligned", kAlign);
    if (b->n_queries == 0) return GOFANN_OK;
    const uint32_t nq = b->n_queries, ng = b->graph_routes.n_routes, npo = b->posting_routes.n_routes;
    const int k = p->topk;
    const int sc = p->search.scorer;

    // ---- query preparation
    gofann_prepared prep{};
    gofann_routes groutes = b->graph_routes;
    if (sc == GOFANN_SCORER_PQ) {
        const int qdt = ix->base_dtype == GOFANN_DTYPE_U8 ? GOFANN_DTYPE_U8 : GOFANN_DTYPE_F32;
        if (l.has_lut) {
            float* lut = at<float>(scratch, l.lut);
            if ((st = gofann_pq_build_lut(b->queries, qdt, nq, ix->dim, ix->pq_centroids, ix->codes.pq_dim, lut,
                                          stream)) != GOFANN_OK)
                return st;
            prep.pq_lut = lut;
        } else {
            prep.pq_query = b->queries;
            prep.pq_centroids = ix->pq_centroids;
            prep.pq_query_dtype = qdt;
            prep.dim = ix->dim;
        }
        prep.n_rows = nq;
    } else {
        const uint32_t pd = ix->codes.padded_dim, na = ix->codes.num_anchors;
        float* rotated = at<float>(scratch, l.rotated);
        void* gemm = at<void>(scratch, l.gemm);
        if ((st = gofann_rabitq_rotate(static_cast<const float*>(b->queries), nq, ix->dim, ix->rq_rotation, pd,
                                       GOFANN_GEMM_TF32X3, rotated, gemm, l.gemm_bytes, status, stream)) != GOFANN_OK)
            return st;
        int8_t* q8 = at<int8_t>(scratch, l.q8);
        float* scale = at<float>(scratch, l.scale);
        float* k1 = at<float>(scratch, l.k1);
        float* gdist = at<float>(scratch, l.gdist);
        if ((st = gofann_rabitq_quantize(rotated, nq, pd, q8, scale, k1, stream)) != GOFANN_OK) return st;
        if ((st = gofann_rabitq_centroid_dist_tc(rotated, nq, ix->rq_anchors, na, pd, GOFANN_GEMM_TF32X3, gdist, gemm,
                                                 l.gemm_bytes, status, stream)) != GOFANN_OK)
            return st;
        if (p->rq_entries && ng) {
            uint32_t* start = at<uint32_t>(scratch, l.start);
            if ((st = gofann_rabitq_route_entries(gdist, na, groutes.query_row, ng, ix->rq_anchor_entry, start,
                                                  stream)) != GOFANN_OK)
                return st;
            groutes.start_local = start;
        }
        prep.rq_q8 = q8;
        prep.rq_scale = scale;
        prep.rq_k1xsumq = k1;
        prep.rq_centroid_dist = gdist;
        prep.n_rows = nq;
    }

    // ---- traversal and posting scans
    uint32_t* g_ids = at<uint32_t>(scratch, l.g_ids);
    float* g_d = at<float>(scratch, l.g_d);
    if (ng) {
        gofann_search_out out{};
        out.ids = g_ids;
        out.dists = g_d;
        out.steps = at<int32_t>(scratch, l.g_steps);
        out.status = status;
        if ((st = gofann_beam_search(&ix->graph, &ix->attrs, &ix->codes, &prep, &groutes, &p->search, &out,
                                     at<void>(scratch, l.beam), l.beam_bytes, stream)) != GOFANN_OK)
            return st;
    }
    uint32_t* p_ids = at<uint32_t>(scratch, l.p_ids);
    float* p_d = at<float>(scratch, l.p_d);
    if (npo) {
        if ((st = gofann_posting_scan(&ix->codes, &prep, &ix->attrs, &b->posting_routes, sc, ix->posting_ids,
                                      b->posting_begin, b->posting_count, p->posting_shortlist, 1, p->search.pq_mode,
                                      p_ids, p_d, status, stream)) != GOFANN_OK)
            return st;
    }

    // ---- exact rerank of both shortlist sets, route -> query merge
    uint32_t* r_ids = at<uint32_t>(scratch, l.r_ids);
    float* r_d = at<float>(scratch, l.r_d);
    const uint32_t n_samples = ix->attrs.n_samples ? ix->attrs.n_samples : ix->codes.n_samples;
    if (ng) {
        if ((st = gofann_rerank(ix->base, ix->base_dtype, n_samples, ix->dim, b->queries, &ix->attrs, &groutes, g_ids,
                                static_cast<uint32_t>(p->search.result_width), k, r_ids, r_d, stream)) != GOFANN_OK)
            return st;
    }
    if (npo) {
        if ((st = gofann_rerank(ix->base, ix->base_dtype, n_samples, ix->dim, b->queries, &ix->attrs,
                                &b->posting_routes, p_ids, static_cast<uint32_t>(p->posting_shortlist), k,
                                r_ids + static_cast<size_t>(ng) * k, r_d + static_cast<size_t>(ng) * k,
                                stream)) != GOFANN_OK)
            return st;
    }
    return gofann_route_merge(r_ids, r_d, static_cast<uint32_t>(k), b->query_route_offsets, b->query_routes, nq, k,
                              out_ids, out_dists, stream);
}

}  // extern "C"
