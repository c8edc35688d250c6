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
