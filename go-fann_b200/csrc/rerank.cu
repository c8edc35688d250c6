// rerank.cu — exact rerank of route shortlists, route -> original-query
// merge, per-shard top-k merge and shard id offsetting.
//
// Rerank keeps the reference's admission rules (highfreq_host_batch_rerank_range,
// src/search/pq/backend_pq.cu:2479-2592; GPU variant 5201-5310): sentinel and
// out-of-range ids dropped, residual label check, duplicates counted once,
// top-k ascending by (dist, id).  One 128-thread block per route: each warp
// computes exact L2 for every 4th candidate (uint8 as exact integers, f32 and
// f16 with fma partials and a butterfly), then warp 0 selects the top-k.
#include "common.cuh"

namespace gofann {
namespace {

constexpr int kRerankWarps = 4;

__device__ __forceinline__ float f16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

template <int kDtype>
__global__ void __launch_bounds__(kRerankWarps * 32) rerank_kernel(
    const void* __restrict__ base, uint32_t n_samples, uint32_t dim, const void* __restrict__ queries,
    AttrView attrs, gofann_routes routes, bool check_labels, const uint32_t* __restrict__ cand, uint32_t width,
    int k, uint32_t* __restrict__ out_ids, float* __restrict__ out_d)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* sd = reinterpret_cast<float*>(smem_raw);
    uint32_t* sid = reinterpret_cast<uint32_t*>(smem_raw + width * 4);
    const uint32_t route = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t row = routes.query_row[route];
    const uint32_t* cr = cand + static_cast<size_t>(route) * width;
    for (uint32_t i = warp; i < width; i += kRerankWarps) {
        uint32_t s = cr[i];
        bool ok = s != kU32Max && s < n_samples;
        if (ok && check_labels) ok = labels_match(routes, attrs, route, s);
        float acc = 0.0f;
        if (ok) {
            if constexpr (kDtype == GOFANN_DTYPE_U8) {
                const uint8_t* b = static_cast<const uint8_t*>(base) + static_cast<size_t>(s) * dim;
                const uint8_t* q = static_cast<const uint8_t*>(queries) + static_cast<size_t>(row) * dim;
                int iacc = 0;
                if ((dim & 3) == 0 && (reinterpret_cast<uintptr_t>(b) & 3) == 0 &&
                    (reinterpret_cast<uintptr_t>(q) & 3) == 0) {
                    const uint32_t* b4 = reinterpret_cast<const uint32_t*>(b);
                    const uint32_t* q4 = reinterpret_cast<const uint32_t*>(q);
                    for (uint32_t w = lane; w < dim / 4; w += 32) {
                        const uint32_t x = __ldg(b4 + w), y = __ldg(q4 + w);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int diff = static_cast<int>((x >> (8 * j)) & 0xff) - static_cast<int>((y >> (8 * j)) & 0xff);
                            iacc += diff * diff;
                        }
                    }
                } else {
                    for (uint32_t d = lane; d < dim; d += 32) {
                        const int diff = static_cast<int>(b[d]) - static_cast<int>(q[d]);
                        iacc += diff * diff;
                    }
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) iacc += __shfl_xor_sync(kFull, iacc, off);
                acc = static_cast<float>(iacc);
            } else {
                const float* q = static_cast<const float*>(queries) + static_cast<size_t>(row) * dim;
                for (uint32_t d = lane; d < dim; d += 32) {
                    float x;
                    if constexpr (kDtype == GOFANN_DTYPE_F32)
                        x = __ldg(static_cast<const float*>(base) + static_cast<size_t>(s) * dim + d);
                    else
                        x = f16_to_f32(__ldg(static_cast<const uint16_t*>(base) + static_cast<size_t>(s) * dim + d));
                    const float diff = __fsub_rn(__ldg(q + d), x);
                    acc = __fmaf_rn(diff, diff, acc);
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(kFull, acc, off));
            }
        } else {
            s = kU32Max;
        }
        if (lane == 0) {
            sd[i] = ok ? acc : FLT_MAX;
            sid[i] = s;
        }
    }
    __syncthreads();
    if (warp == 0)
        warp_select_topk<GOFANN_MAX_TOPK>(
            static_cast<int>(width), k,
            [&](int i, float& x, uint32_t& y) { x = sd[i]; y = sid[i]; },
            out_ids + static_cast<size_t>(route) * k, out_d + static_cast<size_t>(route) * k, lane);
}

constexpr int kMergeWarps = 4;

// One warp per original query; candidates are read in place from the
// routes' shortlists (query_routes lists each query's routes).
__global__ void __launch_bounds__(kMergeWarps * 32) route_merge_kernel(
    const uint32_t* __restrict__ ids, const float* __restrict__ d, uint32_t width,
    const uint32_t* __restrict__ qoff, const uint32_t* __restrict__ qroutes, uint32_t nq, int k,
    uint32_t* __restrict__ out_ids, float* __restrict__ out_d)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t q = blockIdx.x * kMergeWarps + warp;
    if (q >= nq) return;
    const uint32_t r0 = qoff[q], r1 = qoff[q + 1];
    const int total = static_cast<int>((r1 - r0) * width);
    warp_select_topk<GOFANN_MAX_TOPK>(
        total, k,
        [&](int t, float& x, uint32_t& y) {
            const size_t at = static_cast<size_t>(qroutes[r0 + t / width]) * width + t % width;
            y = ids[at];
            x = d[at];
        },
        out_ids + static_cast<size_t>(q) * k, out_d + static_cast<size_t>(q) * k, lane);
}

// Shards hold disjoint ids; layout [n_shards][n_queries][k].
__global__ void __launch_bounds__(kMergeWarps * 32) shard_merge_kernel(
    const uint32_t* __restrict__ ids, const float* __restrict__ d, uint32_t shards, uint32_t nq, int k,
    uint32_t* __restrict__ out_ids, float* __restrict__ out_d)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t q = blockIdx.x * kMergeWarps + warp;
    if (q >= nq) return;
    warp_select_topk<GOFANN_MAX_TOPK>(
        static_cast<int>(shards) * k, k,
        [&](int t, float& x, uint32_t& y) {
            const size_t at = (static_cast<size_t>(t / k) * nq + q) * k + t % k;
            y = ids[at];
            x = d[at];
        },
        out_ids + static_cast<size_t>(q) * k, out_d + static_cast<size_t>(q) * k, lane);
}

__global__ void offset_ids_kernel(uint32_t* ids, size_t n, uint32_t base)
{
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n && ids[i] != kU32Max) ids[i] += base;
}

}  // namespace
}  // namespace gofann

using namespace gofann;

extern "C" {

int gofann_rerank(const void* base, int dtype, uint32_t n_samples, uint32_t dim, const void* queries,
                  const gofann_attrs* attrs, const gofann_routes* routes, const uint32_t* cand_ids, uint32_t width,
                  int32_t topk, uint32_t* out_ids, float* out_dists, void* stream)
{
    if (!base || !queries || !routes || !cand_ids || !out_ids || !out_dists)
        return fail(GOFANN_ERR_INVALID, "rerank: null argument");
    if (!routes->query_row) return fail(GOFANN_ERR_INVALID, "rerank: routes.query_row missing");
    if (topk < 1 || topk > GOFANN_MAX_TOPK)
        return fail(GOFANN_ERR_INVALID, "rerank: topk %d outside 1..%d", topk, GOFANN_MAX_TOPK);
    if (width < 1 || width > GOFANN_MAX_RESULT_WIDTH)
        return fail(GOFANN_ERR_INVALID, "rerank: width %u outside 1..%d", width, GOFANN_MAX_RESULT_WIDTH);
    if (dim == 0) return fail(GOFANN_ERR_INVALID, "rerank: dim is zero");
    const bool check = routes->qlabel_indptr != nullptr;
    if (check && (!attrs || !attrs->label_indptr || !attrs->label_indices))
        return fail(GOFANN_ERR_INVALID, "rerank: residual label check needs the sample label CSR");
    if (routes->n_routes == 0) return GOFANN_OK;
    const AttrView av = make_attr_view(attrs);
    const size_t smem = static_cast<size_t>(width) * 8 + 16;
    cudaStream_t s = as_stream(stream);
    const unsigned blocks = routes->n_routes;
    switch (dtype) {
    case GOFANN_DTYPE_U8:
        rerank_kernel<GOFANN_DTYPE_U8><<<blocks, kRerankWarps * 32, smem, s>>>(base, n_samples, dim, queries, av,
                                                                               *routes, check, cand_ids, width,
                                                                               topk, out_ids, out_dists);
        break;
    case GOFANN_DTYPE_F32:
        rerank_kernel<GOFANN_DTYPE_F32><<<blocks, kRerankWarps * 32, smem, s>>>(base, n_samples, dim, queries, av,
                                                                                *routes, check, cand_ids, width,
                                                                                topk, out_ids, out_dists);
        break;
    case GOFANN_DTYPE_F16:
        rerank_kernel<GOFANN_DTYPE_F16><<<blocks, kRerankWarps * 32, smem, s>>>(base, n_samples, dim, queries, av,
                                                                                *routes, check, cand_ids, width,
                                                                                topk, out_ids, out_dists);
        break;
    default:
        return fail(GOFANN_ERR_INVALID, "rerank: unknown dtype %d", dtype);
    }
    GOFANN_CHECK_LAUNCH("rerank_kernel");
    return GOFANN_OK;
}

int gofann_route_merge(const uint32_t* route_ids, const float* route_dists, uint32_t width,
                       const uint32_t* query_route_offsets, const uint32_t* query_routes, uint32_t n_queries,
                       int32_t topk, uint32_t* out_ids, float* out_dists, void* stream)
{
    if (!route_ids || !route_dists || !query_route_offsets || !query_routes || !out_ids || !out_dists)
        return fail(GOFANN_ERR_INVALID, "route_merge: null argument");
    if (topk < 1 || topk > GOFANN_MAX_TOPK)
        return fail(GOFANN_ERR_INVALID, "route_merge: topk %d outside 1..%d", topk, GOFANN_MAX_TOPK);
    if (width < 1) return fail(GOFANN_ERR_INVALID, "route_merge: width is zero");
    if (n_queries == 0) return GOFANN_OK;
    route_merge_kernel<<<(n_queries + kMergeWarps - 1) / kMergeWarps, kMergeWarps * 32, 0, as_stream(stream)>>>(
        route_ids, route_dists, width, query_route_offsets, query_routes, n_queries, topk, out_ids, out_dists);
    GOFANN_CHECK_LAUNCH("route_merge_kernel");
    return GOFANN_OK;
}

int gofann_shard_merge(const uint32_t* shard_ids, const float* shard_dists, uint32_t n_shards, uint32_t n_queries,
                       int32_t topk, uint32_t* out_ids, float* out_dists, void* stream)
{
    if (!shard_ids || !shard_dists || !out_ids || !out_dists) return fail(GOFANN_ERR_INVALID, "shard_merge: null argument");
    if (topk < 1 || topk > GOFANN_MAX_TOPK)
        return fail(GOFANN_ERR_INVALID, "shard_merge: topk %d outside 1..%d", topk, GOFANN_MAX_TOPK);
    if (n_shards < 1 || n_shards > 64) return fail(GOFANN_ERR_INVALID, "shard_merge: n_shards %u outside 1..64", n_shards);
    if (n_queries == 0) return GOFANN_OK;
    shard_merge_kernel<<<(n_queries + kMergeWarps - 1) / kMergeWarps, kMergeWarps * 32, 0, as_stream(stream)>>>(
        shard_ids, shard_dists, n_shards, n_queries, topk, out_ids, out_dists);
    GOFANN_CHECK_LAUNCH("shard_merge_kernel");
    return GOFANN_OK;
}

int gofann_offset_ids(uint32_t* ids, size_t n, uint32_t base, void* stream)
{
    if (!ids) return fail(GOFANN_ERR_INVALID, "offset_ids: null pointer");
    if (n == 0 || base == 0) return GOFANN_OK;
    offset_ids_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream)>>>(ids, n, base);
    GOFANN_CHECK_LAUNCH("offset_ids_kernel");
    return GOFANN_OK;
}

}  // extern "C"
