// pq.cu — product-quantisation stages: per-query lookup table, ADC scoring
// of (query, sample) pairs, and nearest-centroid encoding.
//
// LUT build follows computePQTable (src/search/pq/backend_pq.cu:1999-2022):
// entry (m, c) = sequential fma(diff, diff, acc) over the subvector with
// diff = q - c.  The B200 kernel keeps one centroid per thread and reuses
// each centroid element across 8 queries staged in shared memory, so the
// centroid table is read once per 8 queries instead of once per query.
#include "pq_device.cuh"

namespace gofann {
namespace {

constexpr int kLutQueriesPerBlock = 8;

template <typename QT>
__global__ void __launch_bounds__(256) pq_lut_kernel(const QT* __restrict__ queries, uint32_t n,
                                                     uint32_t dim, const float* __restrict__ centroids,
                                                     uint32_t pq_dim, float* __restrict__ lut)
{
    extern __shared__ float qs[];  // [kLutQueriesPerBlock][dim]
    const uint32_t q0 = blockIdx.x * kLutQueriesPerBlock;
    const int nq = min(kLutQueriesPerBlock, static_cast<int>(n - q0));
    for (uint32_t i = threadIdx.x; i < static_cast<uint32_t>(nq) * dim; i += blockDim.x)
        qs[i] = static_cast<float>(queries[static_cast<size_t>(q0) * dim + i]);
    __syncthreads();
    const uint32_t c = threadIdx.x;  // one centroid per thread (256 threads)
    const uint32_t w = dim / pq_dim;
    const float* crow = centroids + static_cast<size_t>(c) * dim;
    for (uint32_t m = 0; m < pq_dim; ++m) {
        float acc[kLutQueriesPerBlock];
#pragma unroll
        for (int j = 0; j < kLutQueriesPerBlock; ++j) acc[j] = 0.0f;
        for (uint32_t d = 0; d < w; ++d) {
            const uint32_t k = m * w + d;
            const float cv = __ldg(crow + k);
#pragma unroll
            for (int j = 0; j < kLutQueriesPerBlock; ++j) {
                const float diff = __fsub_rn(qs[j * dim + k], cv);
                acc[j] = __fmaf_rn(diff, diff, acc[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < kLutQueriesPerBlock; ++j)
            if (j < nq)
                lut[(static_cast<size_t>(q0 + j) * pq_dim + m) * GOFANN_PQ_CENTROIDS + c] = acc[j];
    }
}

__global__ void pq_adc_pairs_kernel(const float* __restrict__ lut, uint32_t pq_dim,
                                    const uint8_t* __restrict__ codes,
                                    const uint32_t* __restrict__ pair_row,
                                    const uint32_t* __restrict__ pair_sample, uint32_t n_pairs,
                                    float* __restrict__ out)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_pairs) return;
    const float* row = lut + static_cast<size_t>(pair_row[i]) * pq_dim * GOFANN_PQ_CENTROIDS;
    out[i] = pq_adc_warp_order(row, codes + static_cast<size_t>(pair_sample[i]) * pq_dim, pq_dim);
}

template <typename VT>
__global__ void __launch_bounds__(256) pq_encode_kernel(const VT* __restrict__ vectors, uint32_t n,
                                                        uint32_t dim,
                                                        const float* __restrict__ centroids,
                                                        uint32_t pq_dim, uint8_t* __restrict__ codes)
{
    extern __shared__ float cs[];  // [256][w] centroid slice of subspace m
    const uint32_t m = blockIdx.y;
    const uint32_t w = dim / pq_dim;
    for (uint32_t i = threadIdx.x; i < GOFANN_PQ_CENTROIDS * w; i += blockDim.x)
        cs[i] = centroids[static_cast<size_t>(i / w) * dim + m * w + i % w];
    __syncthreads();
    const uint32_t v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= n) return;
    float x[kMaxEncodeWidth];
#pragma unroll
    for (int d = 0; d < kMaxEncodeWidth; ++d)
        x[d] = d < static_cast<int>(w) ? static_cast<float>(vectors[static_cast<size_t>(v) * dim + m * w + d]) : 0.0f;
    float best = INFINITY;
    uint32_t best_c = 0;
    for (uint32_t c = 0; c < GOFANN_PQ_CENTROIDS; ++c) {
        float acc = 0.0f;
#pragma unroll
        for (int d = 0; d < kMaxEncodeWidth; ++d) {
            if (d < static_cast<int>(w)) {
                const float diff = __fsub_rn(x[d], cs[c * w + d]);
                acc = __fmaf_rn(diff, diff, acc);
            }
        }
        if (acc < best) { best = acc; best_c = c; }
    }
    codes[static_cast<size_t>(v) * pq_dim + m] = static_cast<uint8_t>(best_c);
}

}  // namespace
}  // namespace gofann

using namespace gofann;

extern "C" {

int gofann_pq_build_lut(const void* queries, int query_dtype, uint32_t n, uint32_t dim,
                        const float* centroids, uint32_t pq_dim, float* lut_out, void* stream)
{
    if (!queries || !centroids || !lut_out) return fail(GOFANN_ERR_INVALID, "pq_build_lut: null pointer");
    if (pq_dim == 0 || dim == 0 || dim % pq_dim != 0)
        return fail(GOFANN_ERR_INVALID, "pq_build_lut: dim %u not divisible by pq_dim %u", dim, pq_dim);
    if (n == 0) return GOFANN_OK;
    const size_t smem = static_cast<size_t>(kLutQueriesPerBlock) * dim * sizeof(float);
    if (smem > 200 * 1024) return fail(GOFANN_ERR_UNSUPPORTED, "pq_build_lut: dim %u too large", dim);
    const dim3 grid((n + kLutQueriesPerBlock - 1) / kLutQueriesPerBlock);
    if (query_dtype == GOFANN_DTYPE_U8) {
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(pq_lut_kernel<uint8_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        pq_lut_kernel<uint8_t><<<grid, 256, smem, as_stream(stream)>>>(
            static_cast<const uint8_t*>(queries), n, dim, centroids, pq_dim, lut_out);
    } else if (query_dtype == GOFANN_DTYPE_F32) {
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(pq_lut_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        pq_lut_kernel<float><<<grid, 256, smem, as_stream(stream)>>>(
            static_cast<const float*>(queries), n, dim, centroids, pq_dim, lut_out);
    } else {
        return fail(GOFANN_ERR_INVALID, "pq_build_lut: query dtype must be u8 or f32");
    }
    GOFANN_CHECK_LAUNCH("pq_lut_kernel");
    return GOFANN_OK;
}

int gofann_pq_adc(const float* lut, uint32_t pq_dim, const uint8_t* codes, const uint32_t* pair_row,
                  const uint32_t* pair_sample, uint32_t n_pairs, float* dist_out, void* stream)
{
    if (!lut || !codes || !pair_row || !pair_sample || !dist_out)
        return fail(GOFANN_ERR_INVALID, "pq_adc: null pointer");
    if (pq_dim == 0 || pq_dim > kMaxPqDim)
        return fail(GOFANN_ERR_UNSUPPORTED, "pq_adc: pq_dim %u outside 1..%d", pq_dim, kMaxPqDim);
    if (n_pairs == 0) return GOFANN_OK;
    pq_adc_pairs_kernel<<<(n_pairs + 255) / 256, 256, 0, as_stream(stream)>>>(
        lut, pq_dim, codes, pair_row, pair_sample, n_pairs, dist_out);
    GOFANN_CHECK_LAUNCH("pq_adc_pairs_kernel");
    return GOFANN_OK;
}

int gofann_pq_encode(const void* vectors, int dtype, uint32_t n, uint32_t dim, const float* centroids,
                     uint32_t pq_dim, uint8_t* codes_out, void* stream)
{
    if (!vectors || !centroids || !codes_out) return fail(GOFANN_ERR_INVALID, "pq_encode: null pointer");
    if (pq_dim == 0 || dim % pq_dim != 0 || dim / pq_dim > static_cast<uint32_t>(kMaxEncodeWidth))
        return fail(GOFANN_ERR_UNSUPPORTED, "pq_encode: subvector width must divide dim and be <= %d",
                    kMaxEncodeWidth);
    if (pq_dim > 65535) return fail(GOFANN_ERR_UNSUPPORTED, "pq_encode: pq_dim too large");
    if (n == 0) return GOFANN_OK;
    const uint32_t w = dim / pq_dim;
    const size_t smem = static_cast<size_t>(GOFANN_PQ_CENTROIDS) * w * sizeof(float);
    const dim3 grid((n + 255) / 256, pq_dim);
    if (dtype == GOFANN_DTYPE_U8)
        pq_encode_kernel<uint8_t><<<grid, 256, smem, as_stream(stream)>>>(
            static_cast<const uint8_t*>(vectors), n, dim, centroids, pq_dim, codes_out);
    else if (dtype == GOFANN_DTYPE_F32)
        pq_encode_kernel<float><<<grid, 256, smem, as_stream(stream)>>>(
            static_cast<const float*>(vectors), n, dim, centroids, pq_dim, codes_out);
    else
        return fail(GOFANN_ERR_INVALID, "pq_encode: dtype must be u8 or f32");
    GOFANN_CHECK_LAUNCH("pq_encode_kernel");
    return GOFANN_OK;
}

}  // extern "C"
