// rabitq.cu — RaBitQ query preparation and the pairwise 1-bit estimator.
//
// Quantisation follows quantize_rabitq_queries_int8_kernel and
// compute_rabitq_query_factors_kernel (src/search/rabitq/backend_rabitq.cu:
// 2898-2964): scale = max|q|/127 (1 when zero), q8 = clamp(rint(q/scale),
// -127, 127) with round-half-even, k1xsumq = -0.5 * sum(q).  One 256-thread
// block per query does both in one pass over the rotated row.
#include "rq_device.cuh"

namespace gofann {
namespace {

__global__ void __launch_bounds__(256) rq_quantize_kernel(const float* __restrict__ rotated, uint32_t n,
                                                          uint32_t padded_dim, int8_t* __restrict__ q8,
                                                          float* __restrict__ scale_out,
                                                          float* __restrict__ k1_out)
{
    __shared__ float part[256];
    __shared__ float mx_part[256];
    const uint32_t q = blockIdx.x;
    const float* src = rotated + static_cast<size_t>(q) * padded_dim;
    float s = 0.0f, mx = 0.0f;
    for (uint32_t d = threadIdx.x; d < padded_dim; d += 256) {
        const float v = src[d];
        s = __fadd_rn(s, v);
        mx = fmaxf(mx, fabsf(v));
    }
    part[threadIdx.x] = s;
    mx_part[threadIdx.x] = mx;
    __syncthreads();
    for (int stride = 128; stride > 0; stride >>= 1) {
        if (threadIdx.x < stride) {
            part[threadIdx.x] = __fadd_rn(part[threadIdx.x], part[threadIdx.x + stride]);
            mx_part[threadIdx.x] = fmaxf(mx_part[threadIdx.x], mx_part[threadIdx.x + stride]);
        }
        __syncthreads();
    }
    const float m = mx_part[0];
    const float scale = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
    if (threadIdx.x == 0) {
        scale_out[q] = scale;
        k1_out[q] = __fmul_rn(part[0], -0.5f);
    }
    for (uint32_t d = threadIdx.x; d < padded_dim; d += 256) {
        const int v = max(-127, min(127, __float2int_rn(__fdiv_rn(src[d], scale))));
        q8[static_cast<size_t>(q) * padded_dim + d] = static_cast<int8_t>(v);
    }
}

// gdist[q][a] = sum_d (q_d - c_a,d)^2, sequential fma per anchor (the
// direct form of compute_rabitq_centroid_distances_kernel,
// backend_rabitq.cu:2966-2999); tolerance-checked against FP64.
__global__ void __launch_bounds__(256) rq_centroid_dist_kernel(const float* __restrict__ rotated,
                                                               const float* __restrict__ anchors,
                                                               uint32_t num_anchors, uint32_t padded_dim,
                                                               float* __restrict__ gdist)
{
    extern __shared__ float qs[];
    const uint32_t q = blockIdx.x;
    for (uint32_t d = threadIdx.x; d < padded_dim; d += blockDim.x)
        qs[d] = rotated[static_cast<size_t>(q) * padded_dim + d];
    __syncthreads();
    // one warp per anchor, lanes over dimensions, butterfly reduce
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (uint32_t a = blockIdx.y * 8 + warp; a < num_anchors; a += gridDim.y * 8) {
        const float* c = anchors + static_cast<size_t>(a) * padded_dim;
        float acc = 0.0f;
        for (uint32_t d = lane; d < padded_dim; d += 32) {
            const float diff = __fsub_rn(qs[d], __ldg(c + d));
            acc = __fmaf_rn(diff, diff, acc);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(kFull, acc, off));
        if (lane == 0) gdist[static_cast<size_t>(q) * num_anchors + a] = acc;
    }
}

// 1-bit RaBitQ encoder (index time; the quantizer of the reference's RaBitQ
// artefacts, third_party/cuvs_rabitq/.../quantizer_gpu_fast.cu:180-270, with
// the MSB-first packing of quantizer_gpu.cu:31-46): one warp per vector.  For
// the residual r = (x - c) R and the rotated centroid c of its anchor, bit d
// = (r_d > 0), xu_d = bit - 1/2, and over the padded dimensions
//   rr = sum r^2, rxu = sum r xu, cxu = sum c xu, xuxu = P / 4:
//   f_add = rr + 2 rr cxu / rxu,  f_rescale = -2 rr / rxu,
//   f_err = 2 * 1.9 * sqrt(rr) * sqrt(max(0, (rr xuxu / rxu^2 - 1) / (P - 1)))
// (rxu = 0 is replaced by 1e-30).  FP32 throughout in a fixed order: lane l
// accumulates dimensions l, l + 32, ... (rr by fma), the lane partials are
// combined by an xor butterfly 16..1, and the factor formulas run as written
// left to right with correctly rounded division and square root.  Code word
// w holds dimensions 32w..32w+31 with dimension 32w+j at bit 31-j: the
// bit-reversed ballot of the lanes' bits.
__global__ void __launch_bounds__(256) rq_encode_kernel(const float* __restrict__ residual,
                                                        const float* __restrict__ rotated_centroids,
                                                        const uint32_t* __restrict__ anchor_ids, uint32_t n,
                                                        uint32_t padded_dim, uint32_t* __restrict__ codes,
                                                        float* __restrict__ factors)
{
    const uint32_t v = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (v >= n) return;
    const float* r = residual + static_cast<size_t>(v) * padded_dim;
    const float* c = rotated_centroids + static_cast<size_t>(anchor_ids[v]) * padded_dim;
    uint32_t* code = codes + static_cast<size_t>(v) * (padded_dim / 32);
    float rr = 0.0f, rxu = 0.0f, cxu = 0.0f;
    for (uint32_t w = 0; w < padded_dim / 32; ++w) {
        const uint32_t d = w * 32 + lane;
        const float x = r[d];
        const bool bit = x > 0.0f;
        const float xu = bit ? 0.5f : -0.5f;
        rr = __fmaf_rn(x, x, rr);
        rxu = __fadd_rn(rxu, __fmul_rn(x, xu));
        cxu = __fadd_rn(cxu, __fmul_rn(c[d], xu));
        const unsigned b = __ballot_sync(kFull, bit);
        if (lane == 0) code[w] = __brev(b);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        rr = __fadd_rn(rr, __shfl_xor_sync(kFull, rr, off));
        rxu = __fadd_rn(rxu, __shfl_xor_sync(kFull, rxu, off));
        cxu = __fadd_rn(cxu, __shfl_xor_sync(kFull, cxu, off));
    }
    if (lane == 0) {
        const float xuxu = __fmul_rn(static_cast<float>(padded_dim), 0.25f);
        if (rxu == 0.0f) rxu = 1e-30f;
        float* f = factors + static_cast<size_t>(v) * 3;
        f[0] = __fadd_rn(rr, __fdiv_rn(__fmul_rn(__fmul_rn(2.0f, rr), cxu), rxu));
        f[1] = __fdiv_rn(__fmul_rn(-2.0f, rr), rxu);
        float t = __fdiv_rn(__fsub_rn(__fdiv_rn(__fmul_rn(rr, xuxu), __fmul_rn(rxu, rxu)), 1.0f),
                            static_cast<float>(padded_dim - 1));
        if (!(t > 0.0f)) t = 0.0f;
        f[2] = __fmul_rn(__fmul_rn(3.8f, __fsqrt_rn(rr)), __fsqrt_rn(t));
    }
}

// Entry rows of graph routes from the centroid distances: one warp per
// route takes the anchor of smallest distance (lowest index on ties) and
// starts the route at that anchor's entry row.
__global__ void __launch_bounds__(256) rq_entries_kernel(const float* __restrict__ gdist, uint32_t num_anchors,
                                                         const uint32_t* __restrict__ query_row, uint32_t n_routes,
                                                         const uint32_t* __restrict__ anchor_entry,
                                                         uint32_t* __restrict__ start_out)
{
    const uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n_routes) return;
    const float* g = gdist + static_cast<size_t>(query_row[r]) * num_anchors;
    float bd = FLT_MAX;
    uint32_t bi = kU32Max;
    for (uint32_t a = lane; a < num_anchors; a += 32) {
        const float d = g[a];
        if (bi == kU32Max || d < bd) { bd = d; bi = a; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float od = __shfl_xor_sync(kFull, bd, off);
        const uint32_t oi = __shfl_xor_sync(kFull, bi, off);
        if (oi != kU32Max && (bi == kU32Max || od < bd || (od == bd && oi < bi))) { bd = od; bi = oi; }
    }
    if (lane == 0) start_out[r] = bi == kU32Max ? 0u : anchor_entry[bi];
}

// One warp per pair: lanes split the code words; the integer partials are
// exact, then the combine runs on lane 0.
__global__ void rq_score_pairs_kernel(gofann_codes codes, gofann_prepared prep,
                                      const uint32_t* __restrict__ pair_row,
                                      const uint32_t* __restrict__ pair_sample, uint32_t n_pairs,
                                      float* __restrict__ out, int32_t* __restrict__ ip_out)
{
    const uint32_t warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp_global >= n_pairs) return;
    const uint32_t row = pair_row[warp_global], sample = pair_sample[warp_global];
    const uint32_t words = codes.padded_dim / 32;
    const uint32_t* cw = reinterpret_cast<const uint32_t*>(codes.rq_codes + static_cast<size_t>(sample) * (codes.padded_dim / 8));
    const int8_t* q8 = prep.rq_q8 + static_cast<size_t>(row) * codes.padded_dim;
    int32_t acc = 0;
    for (uint32_t w = lane; w < words; w += 32) {
        uint32_t x = cw[w];
        while (x) {
            const int k = __clz(x);  // set bit 31-k <-> dimension 32w+k
            acc += q8[w * 32 + k];
            x &= ~(0x80000000u >> k);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(kFull, acc, off);
    if (lane == 0) {
        const uint32_t anchor = codes.rq_anchor_ids[sample];
        out[warp_global] = rq_combine(acc, prep.rq_scale[row], prep.rq_k1xsumq[row],
                                      codes.rq_factors[static_cast<size_t>(sample) * 3],
                                      codes.rq_factors[static_cast<size_t>(sample) * 3 + 1],
                                      prep.rq_centroid_dist[static_cast<size_t>(row) * codes.num_anchors + anchor]);
        if (ip_out) ip_out[warp_global] = acc;
    }
}

}  // namespace
}  // namespace gofann

using namespace gofann;

extern "C" {

int gofann_rabitq_quantize(const float* rotated, uint32_t n, uint32_t padded_dim, int8_t* q8_out,
                           float* scale_out, float* k1xsumq_out, void* stream)
{
    if (!rotated || !q8_out || !scale_out || !k1xsumq_out)
        return fail(GOFANN_ERR_INVALID, "rabitq_quantize: null pointer");
    if (padded_dim == 0 || padded_dim % 64 != 0)
        return fail(GOFANN_ERR_INVALID, "rabitq_quantize: padded_dim %u must be a positive multiple of 64",
                    padded_dim);
    if (n == 0) return GOFANN_OK;
    rq_quantize_kernel<<<n, 256, 0, as_stream(stream)>>>(rotated, n, padded_dim, q8_out, scale_out, k1xsumq_out);
    GOFANN_CHECK_LAUNCH("rq_quantize_kernel");
    return GOFANN_OK;
}

int gofann_rabitq_centroid_dist(const float* rotated, uint32_t n, const float* anchors, uint32_t num_anchors,
                                uint32_t padded_dim, float* gdist_out, void* stream)
{
    if (!rotated || !anchors || !gdist_out) return fail(GOFANN_ERR_INVALID, "rabitq_centroid_dist: null pointer");
    if (padded_dim == 0 || padded_dim > 4096)
        return fail(GOFANN_ERR_UNSUPPORTED, "rabitq_centroid_dist: padded_dim %u outside 1..4096", padded_dim);
    if (n == 0 || num_anchors == 0) return GOFANN_OK;
    const uint32_t ay = min(64u, (num_anchors + 7) / 8);
    const size_t smem = static_cast<size_t>(padded_dim) * sizeof(float);
    rq_centroid_dist_kernel<<<dim3(n, ay), 256, smem, as_stream(stream)>>>(rotated, anchors, num_anchors,
                                                                           padded_dim, gdist_out);
    GOFANN_CHECK_LAUNCH("rq_centroid_dist_kernel");
    return GOFANN_OK;
}

int gofann_rabitq_encode(const float* residual, const float* rotated_centroids, const uint32_t* anchor_ids,
                         uint32_t n, uint32_t padded_dim, uint8_t* codes_out, float* factors_out, void* stream)
{
    if (!residual || !rotated_centroids || !anchor_ids || !codes_out || !factors_out)
        return fail(GOFANN_ERR_INVALID, "rabitq_encode: null pointer");
    if (padded_dim < 64 || padded_dim % 64 != 0)
        return fail(GOFANN_ERR_INVALID, "rabitq_encode: padded_dim %u must be a positive multiple of 64", padded_dim);
    if ((reinterpret_cast<uintptr_t>(codes_out) & 3) != 0)
        return fail(GOFANN_ERR_INVALID, "rabitq_encode: codes must be 4-byte aligned");
    if (n == 0) return GOFANN_OK;
    const uint64_t threads = static_cast<uint64_t>(n) * 32;
    rq_encode_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, as_stream(stream)>>>(
        residual, rotated_centroids, anchor_ids, n, padded_dim, reinterpret_cast<uint32_t*>(codes_out), factors_out);
    GOFANN_CHECK_LAUNCH("rq_encode_kernel");
    return GOFANN_OK;
}

int gofann_rabitq_route_entries(const float* gdist, uint32_t num_anchors, const uint32_t* query_row, uint32_t n_routes,
                                const uint32_t* anchor_entry, uint32_t* start_local_out, void* stream)
{
    if (!gdist || !query_row || !anchor_entry || !start_local_out)
        return fail(GOFANN_ERR_INVALID, "rabitq_route_entries: null pointer");
    if (num_anchors == 0) return fail(GOFANN_ERR_INVALID, "rabitq_route_entries: no anchors");
    if (n_routes == 0) return GOFANN_OK;
    const uint64_t threads = static_cast<uint64_t>(n_routes) * 32;
    rq_entries_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, as_stream(stream)>>>(
        gdist, num_anchors, query_row, n_routes, anchor_entry, start_local_out);
    GOFANN_CHECK_LAUNCH("rq_entries_kernel");
    return GOFANN_OK;
}

int gofann_rabitq_score(const gofann_codes* codes, const gofann_prepared* prep, const uint32_t* pair_row,
                        const uint32_t* pair_sample, uint32_t n_pairs, float* dist_out, int32_t* ip_out,
                        void* stream)
{
    if (!codes || !prep || !pair_row || !pair_sample || !dist_out)
        return fail(GOFANN_ERR_INVALID, "rabitq_score: null pointer");
    if (!codes->rq_codes || !codes->rq_factors || !codes->rq_anchor_ids || !prep->rq_q8 || !prep->rq_scale ||
        !prep->rq_k1xsumq || !prep->rq_centroid_dist)
        return fail(GOFANN_ERR_INVALID, "rabitq_score: RaBitQ arrays missing");
    if (codes->padded_dim == 0 || codes->padded_dim % 64 != 0 || codes->padded_dim > 4096)
        return fail(GOFANN_ERR_UNSUPPORTED, "rabitq_score: padded_dim %u unsupported", codes->padded_dim);
    if (n_pairs == 0) return GOFANN_OK;
    const uint64_t threads = static_cast<uint64_t>(n_pairs) * 32;
    rq_score_pairs_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, as_stream(stream)>>>(
        *codes, *prep, pair_row, pair_sample, n_pairs, dist_out, ip_out);
    GOFANN_CHECK_LAUNCH("rq_score_pairs_kernel");
    return GOFANN_OK;
}

}  // extern "C"
