// posting.cu — brute-force scans of low-frequency label postings (and any
// explicit candidate slice), fused DNF filter, top-shortlist by (dist, id).
//
// The reference scans one route per single-thread block, inserting into a
// (dist, id) max-heap one candidate at a time (lowfreq_pq_scan_kernel,
// src/search/pq/backend_pq.cu:2046-2185; RaBitQ twin backend_rabitq.cu:
// 5396-5751).  With unique candidate ids that heap ends holding exactly the
// k smallest (dist, id) pairs of the passing candidates, whatever the
// insertion order, and score-first elision only skips candidates that cannot
// enter.  So here one 256-thread block per route scores a chunk of
// candidates in parallel into shared memory and a bitonic sort keeps the k
// best; the PQ LUT (or RaBitQ bit planes) is staged in shared memory once
// per route.  PQ distances keep the reference's sequential subspace order.
#include "pq_device.cuh"
#include "rq_device.cuh"

namespace gofann {
namespace {

constexpr int kScanThreads = 256;
constexpr int kSortSize = 4096;          // pairs per sort round
constexpr int kKeep = 512;               // slots reserved for the running top-k (>= 400)
constexpr int kChunk = kSortSize - kKeep;

__device__ __forceinline__ void bitonic_sort_pairs(float* d, uint32_t* id, int n, int tid, int nthreads)
{
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < n / 2; i += nthreads) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = (lo & size) == 0;
                const float dl = d[lo], dh = d[hi];
                const uint32_t il = id[lo], ih = id[hi];
                const bool greater = pair_less(dh, ih, dl, il);  // lo > hi
                if (greater == up) { d[lo] = dh; d[hi] = dl; id[lo] = ih; id[hi] = il; }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ uint32_t next_pow2(uint32_t x)
{
    return x <= 1 ? 1u : 1u << (32 - __clz(x - 1));
}

// One block per route (the hardware balances routes of very different
// lengths); the sort spans only as many slots as the route has candidates.
template <int kScorer>
__global__ void __launch_bounds__(kScanThreads) posting_scan_kernel(
    gofann_codes codes, gofann_prepared prep, AttrView attrs, gofann_routes routes,
    const uint32_t* __restrict__ posting_ids, const uint64_t* __restrict__ route_begin,
    const uint32_t* __restrict__ route_count, int k, uint32_t* __restrict__ out_ids, float* __restrict__ out_d)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* sd = reinterpret_cast<float*>(smem_raw);
    uint32_t* sid = reinterpret_cast<uint32_t*>(smem_raw + kSortSize * sizeof(float));
    float* table = reinterpret_cast<float*>(smem_raw + kSortSize * (sizeof(float) + sizeof(uint32_t)));
    const int tid = threadIdx.x;
    const int pq_dim = static_cast<int>(codes.pq_dim);
    {
        const uint32_t route = blockIdx.x;
        const uint32_t row = routes.query_row[route];
        const bool pred_on = pred_enabled(routes, route);
        RqQueryView rq{};
        if constexpr (kScorer == GOFANN_SCORER_PQ) {
            const int dim = static_cast<int>(prep.dim);
            if (prep.pq_lut) {
                const float4* g = reinterpret_cast<const float4*>(prep.pq_lut + static_cast<size_t>(row) * pq_dim *
                                                                                    GOFANN_PQ_CENTROIDS);
                float4* t4 = reinterpret_cast<float4*>(table);
                for (int i = tid; i < pq_dim * GOFANN_PQ_CENTROIDS / 4; i += kScanThreads) t4[i] = __ldg(g + i);
            } else {
                // fused table build (computePQTable, backend_pq.cu:1999-2022, which
                // the reference also runs inside its scan): query row to shared
                // memory, then thread c evaluates column c of every subspace
                float* q = table + pq_dim * GOFANN_PQ_CENTROIDS;
                if (prep.pq_query_dtype == GOFANN_DTYPE_U8) {
                    const uint8_t* qr = static_cast<const uint8_t*>(prep.pq_query) + static_cast<size_t>(row) * dim;
                    for (int i = tid; i < dim; i += kScanThreads) q[i] = static_cast<float>(qr[i]);
                } else {
                    const float* qr = static_cast<const float*>(prep.pq_query) + static_cast<size_t>(row) * dim;
                    for (int i = tid; i < dim; i += kScanThreads) q[i] = qr[i];
                }
                __syncthreads();
                const int w = dim / pq_dim;
                const float* crow = prep.pq_centroids + static_cast<size_t>(tid) * dim;  // kScanThreads == 256
                const uint64_t keep = l2_keep_policy();  // the codebook is shared by every route
                for (int m = 0; m < pq_dim; ++m)
                    table[m * GOFANN_PQ_CENTROIDS + tid] = pq_entry<0>(q + m * w, crow + m * w, w, keep);
            }
        } else {
            rq_build_planes(prep.rq_q8 + static_cast<size_t>(row) * codes.padded_dim,
                            static_cast<int>(codes.padded_dim), reinterpret_cast<uint32_t*>(table), tid,
                            kScanThreads);
            rq.planes = reinterpret_cast<const uint32_t*>(table);
            rq.scale = prep.rq_scale[row];
            rq.k1 = prep.rq_k1xsumq[row];
            rq.gdist = prep.rq_centroid_dist + static_cast<size_t>(row) * codes.num_anchors;
        }
        const uint64_t begin = route_begin[route];
        const uint32_t count = route_count[route];
        // one chunk: candidates at [0, count), the sort spans the next power of
        // two; several: the running top-k at [0, kKeep), chunks after it
        const bool single = count <= static_cast<uint32_t>(kChunk);
        const int keep_slots = single ? 0 : kKeep;
        const int chunk = single ? static_cast<int>(count) : kChunk;
        const int n_sort = single ? static_cast<int>(next_pow2(count)) : kSortSize;
        for (int i = tid; i < keep_slots; i += kScanThreads) { sd[i] = FLT_MAX; sid[i] = kU32Max; }
        __syncthreads();
        for (uint32_t c0 = 0; c0 < count; c0 += static_cast<uint32_t>(chunk)) {
            for (int j = tid; j < n_sort - keep_slots; j += kScanThreads) {
                const uint32_t i = c0 + j;
                float dist = FLT_MAX;
                uint32_t s = kU32Max;
                if (j < chunk && i < count) {
                    s = posting_ids[begin + i];
                    if (s != kU32Max && pred_on && !pred_matches(routes, attrs, route, s)) s = kU32Max;
                    if (s != kU32Max) {
                        if constexpr (kScorer == GOFANN_SCORER_PQ) {
                            dist = pq_adc_sequential(table, codes.pq_codes + static_cast<size_t>(s) * pq_dim,
                                                     pq_dim);
                        } else {
                            dist = rq_estimate(codes, rq, s);
                        }
                    }
                }
                sd[keep_slots + j] = s == kU32Max ? FLT_MAX : dist;
                sid[keep_slots + j] = s;
            }
            __syncthreads();
            bitonic_sort_pairs(sd, sid, n_sort, tid, kScanThreads);
        }
        for (int i = tid; i < k; i += kScanThreads) {
            const bool have = i < n_sort && count > 0;
            const uint32_t id = have ? sid[i] : kU32Max;
            out_ids[static_cast<size_t>(route) * k + i] = id;
            out_d[static_cast<size_t>(route) * k + i] = id == kU32Max ? FLT_MAX : sd[i];
        }
    }
}

}  // namespace
}  // namespace gofann

using namespace gofann;

extern "C" {

int gofann_posting_scan(const gofann_codes* codes, const gofann_prepared* prep, const gofann_attrs* attrs,
                        const gofann_routes* routes, int scorer, const uint32_t* posting_ids,
                        const uint64_t* route_begin, const uint32_t* route_count, int32_t shortlist_k,
                        int32_t score_first, uint32_t* out_ids, float* out_dists, void* stream)
{
    (void)score_first;  // identical results either way (see file comment)
    if (!codes || !prep || !routes || !posting_ids || !route_begin || !route_count || !out_ids || !out_dists)
        return fail(GOFANN_ERR_INVALID, "posting_scan: null argument");
    if (shortlist_k < 1 || shortlist_k > GOFANN_MAX_SHORTLIST)
        return fail(GOFANN_ERR_INVALID, "posting_scan: shortlist %d outside 1..%d", shortlist_k, GOFANN_MAX_SHORTLIST);
    if (!routes->query_row) return fail(GOFANN_ERR_INVALID, "posting_scan: routes.query_row missing");
    if (routes->pred_offsets && (!attrs || !attrs->label_indptr || !routes->clauses || !routes->pred_handles))
        return fail(GOFANN_ERR_INVALID, "posting_scan: predicate arrays missing");
    if (routes->n_routes == 0) return GOFANN_OK;
    AttrView av{};
    if (attrs) {
        av.indptr = attrs->label_indptr;
        av.indices = attrs->label_indices;
        av.ranges = attrs->range_values;
        av.n_samples = attrs->n_samples;
        av.range_count = attrs->range_count;
    }
    size_t table_bytes = 0;
    if (scorer == GOFANN_SCORER_PQ) {
        if (!codes->pq_codes) return fail(GOFANN_ERR_INVALID, "posting_scan: PQ codes missing");
        if (codes->pq_dim == 0 || codes->pq_dim > static_cast<uint32_t>(kMaxPqDim))
            return fail(GOFANN_ERR_UNSUPPORTED, "posting_scan: pq_dim %u unsupported", codes->pq_dim);
        table_bytes = static_cast<size_t>(codes->pq_dim) * GOFANN_PQ_CENTROIDS * sizeof(float);
        if (!prep->pq_lut) {
            if (!prep->pq_query || !prep->pq_centroids || prep->dim == 0 || prep->dim % codes->pq_dim != 0 ||
                prep->dim > 4096)
                return fail(GOFANN_ERR_INVALID, "posting_scan: needs pq_lut, or pq_query + pq_centroids + dim");
            table_bytes += static_cast<size_t>(prep->dim) * sizeof(float);
        }
    } else if (scorer == GOFANN_SCORER_RABITQ) {
        if (!codes->rq_codes || !prep->rq_q8) return fail(GOFANN_ERR_INVALID, "posting_scan: RaBitQ arrays missing");
        if (codes->padded_dim == 0 || codes->padded_dim % 64 != 0 || codes->padded_dim > 4096)
            return fail(GOFANN_ERR_UNSUPPORTED, "posting_scan: padded_dim %u unsupported", codes->padded_dim);
        table_bytes = static_cast<size_t>(codes->padded_dim);
    } else {
        return fail(GOFANN_ERR_INVALID, "posting_scan: unknown scorer %d", scorer);
    }
    const size_t smem = static_cast<size_t>(kSortSize) * 8 + table_bytes;
    cudaStream_t s = as_stream(stream);
    const auto kern = scorer == GOFANN_SCORER_PQ ? posting_scan_kernel<GOFANN_SCORER_PQ>
                                                 : posting_scan_kernel<GOFANN_SCORER_RABITQ>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e, "posting_scan: shared memory attribute");
    kern<<<routes->n_routes, kScanThreads, smem, s>>>(*codes, *prep, av, *routes, posting_ids, route_begin,
                                                      route_count, shortlist_k, out_ids, out_dists);
    GOFANN_CHECK_LAUNCH("posting_scan_kernel");
    return GOFANN_OK;
}

}  // extern "C"
