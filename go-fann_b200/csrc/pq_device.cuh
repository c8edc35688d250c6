// pq_device.cuh — device-side PQ scoring used by the pair kernel, the
// traversal and the posting scans.
#pragma once

#include "common.cuh"

namespace gofann {

constexpr int kMaxPqDim = 128;
constexpr int kMaxEncodeWidth = 32;

// Loads a code row of `m_bytes` (<= 128) bytes into 32-bit words, with
// 16-byte vector loads when the row is 16-byte aligned and sized.
__device__ __forceinline__ void load_code_words(const uint8_t* __restrict__ code, int m_bytes,
                                                uint32_t (&cw)[kMaxPqDim / 4])
{
    if ((m_bytes & 15) == 0 && (reinterpret_cast<uintptr_t>(code) & 15) == 0) {
        const uint4* p = reinterpret_cast<const uint4*>(code);
#pragma unroll
        for (int i = 0; i < kMaxPqDim / 16; ++i) {
            if (i < (m_bytes >> 4)) {
                const uint4 x = __ldg(p + i);
                cw[4 * i + 0] = x.x; cw[4 * i + 1] = x.y; cw[4 * i + 2] = x.z; cw[4 * i + 3] = x.w;
            } else {
                cw[4 * i + 0] = cw[4 * i + 1] = cw[4 * i + 2] = cw[4 * i + 3] = 0;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < kMaxPqDim / 4; ++i) {
            uint32_t word = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b)
                if (4 * i + b < m_bytes) word |= static_cast<uint32_t>(__ldg(code + 4 * i + b)) << (8 * b);
            cw[i] = word;
        }
    }
}

__device__ __forceinline__ uint32_t code_byte(const uint32_t (&cw)[kMaxPqDim / 4], int m)
{
    return (cw[m >> 2] >> ((m & 3) * 8)) & 0xffu;
}

// ADC in the reference's warp order (backend_pq.cu:4711-4725), computed by
// one thread: lane j's partial sums subspaces j, j+32, ... from 0, then the
// xor butterfly.  `lut_row` is [pq_dim][256] in global or shared memory.
__device__ __forceinline__ float pq_adc_words(const float* lut_row, const uint32_t (&cw)[kMaxPqDim / 4],
                                              int pq_dim)
{
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.0f;
#pragma unroll
    for (int m = 0; m < kMaxPqDim; ++m)
        if (m < pq_dim) v[m & 31] = __fadd_rn(v[m & 31], lut_row[m * GOFANN_PQ_CENTROIDS + code_byte(cw, m)]);
    return butterfly_sum32(v);
}

__device__ __forceinline__ float pq_adc_warp_order(const float* lut_row, const uint8_t* code, int pq_dim)
{
    uint32_t cw[kMaxPqDim / 4];
    load_code_words(code, pq_dim, cw);
    return pq_adc_words(lut_row, cw, pq_dim);
}

// Posting-scan order: sequential over subspaces (backend_pq.cu:2101-2104).
__device__ __forceinline__ float pq_adc_sequential(const float* lut_row, const uint8_t* code, int pq_dim)
{
    uint32_t cw[kMaxPqDim / 4];
    load_code_words(code, pq_dim, cw);
    float d = 0.0f;
#pragma unroll
    for (int m = 0; m < kMaxPqDim; ++m)
        if (m < pq_dim) d = __fadd_rn(d, lut_row[m * GOFANN_PQ_CENTROIDS + code_byte(cw, m)]);
    return d;
}

}  // namespace gofann
