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

// Code row of at most kMaxM bytes with an L2 policy (code rows are streaming
// data), into kMaxM / 4 words.
template <int kMaxM>
__device__ __forceinline__ void load_code_words(const uint8_t* __restrict__ code, int m_bytes,
                                                uint32_t (&cw)[kMaxM / 4], uint64_t pol)
{
    if ((m_bytes & 15) == 0 && (reinterpret_cast<uintptr_t>(code) & 15) == 0) {
        const uint4* p = reinterpret_cast<const uint4*>(code);
#pragma unroll
        for (int i = 0; i < kMaxM / 16; ++i) {
            if (i < (m_bytes >> 4)) {
                const uint4 x = ldg_u32x4(p + i, pol);
                cw[4 * i + 0] = x.x; cw[4 * i + 1] = x.y; cw[4 * i + 2] = x.z; cw[4 * i + 3] = x.w;
            } else {
                cw[4 * i + 0] = cw[4 * i + 1] = cw[4 * i + 2] = cw[4 * i + 3] = 0;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < kMaxM / 4; ++i) {
            uint32_t word = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b)
                if (4 * i + b < m_bytes) word |= static_cast<uint32_t>(__ldg(code + 4 * i + b)) << (8 * b);
            cw[i] = word;
        }
    }
}

template <int kWords>
__device__ __forceinline__ uint32_t code_byte(const uint32_t (&cw)[kWords], int m)
{
    return (cw[m >> 2] >> ((m & 3) * 8)) & 0xffu;
}


// ADC in the reference's warp order (backend_pq.cu:4711-4725), computed by
// one thread: lane j's partial sums subspaces j, j+32, ... from 0, then the
// xor butterfly.  `lut_row` is [pq_dim][256] in global or shared memory.
template <int kMaxM>
__device__ __forceinline__ float pq_adc_words(const float* lut_row, const uint32_t (&cw)[kMaxM / 4], int pq_dim)
{
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.0f;
#pragma unroll
    for (int m = 0; m < kMaxM; ++m)
        if (m < pq_dim) v[m & 31] = __fadd_rn(v[m & 31], lut_row[m * GOFANN_PQ_CENTROIDS + code_byte(cw, m)]);
    return butterfly_sum32(v);
}

// pq_adc_words over a table row in global memory, table gathers under the
// `keep` L2 policy.
template <int kMaxM>
__device__ __forceinline__ float pq_adc_words_global(const float* __restrict__ lut_row,
                                                     const uint32_t (&cw)[kMaxM / 4], int pq_dim, uint64_t keep)
{
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.0f;
#pragma unroll
    for (int m = 0; m < kMaxM; ++m)
        if (m < pq_dim)
            v[m & 31] = __fadd_rn(v[m & 31], ldg_f32(lut_row + m * GOFANN_PQ_CENTROIDS + code_byte(cw, m), keep));
    return butterfly_sum32(v);
}

__device__ __forceinline__ float pq_adc_warp_order(const float* lut_row, const uint8_t* code, int pq_dim)
{
    uint32_t cw[kMaxPqDim / 4];
    load_code_words(code, pq_dim, cw);
    return pq_adc_words<kMaxPqDim>(lut_row, cw, pq_dim);
}

// Table entry (m, c) = sum over the subvector of fma(diff, diff, acc), diff =
// q - c, sequential (computePQTable, backend_pq.cu:1999-2022).  `q` is the
// query subvector (shared memory), `cr` the centroid subvector (global).
template <int kW>
__device__ __forceinline__ float pq_entry(const float* q, const float* __restrict__ cr, int w, uint64_t keep)
{
    float acc = 0.0f;
    if constexpr (kW == 4) {
        const float4 c = ldg_f32x4(reinterpret_cast<const float4*>(cr), keep);
        float d = __fsub_rn(q[0], c.x);
        acc = __fmaf_rn(d, d, acc);
        d = __fsub_rn(q[1], c.y);
        acc = __fmaf_rn(d, d, acc);
        d = __fsub_rn(q[2], c.z);
        acc = __fmaf_rn(d, d, acc);
        d = __fsub_rn(q[3], c.w);
        acc = __fmaf_rn(d, d, acc);
    } else {
        for (int d = 0; d < w; ++d) {
            const float diff = __fsub_rn(q[d], ldg_f32(cr + d, keep));
            acc = __fmaf_rn(diff, diff, acc);
        }
    }
    return acc;
}

// ADC in the reference's warp order with every table entry evaluated from
// the query (shared memory, [dim] floats) and the codebook ([256][dim],
// global, L1/L2-resident since all routes share it) instead of read from a
// per-query table: same operations in the same order, so the same bits, and
// no 48 KB table per in-flight query.
template <int kW, int kMaxM>
__device__ __forceinline__ float pq_adc_direct(const float* q, const float* __restrict__ cent, int dim,
                                               const uint8_t* code, int pq_dim, uint64_t keep, uint64_t stream)
{
    uint32_t cw[kMaxM / 4];
    load_code_words<kMaxM>(code, pq_dim, cw, stream);
    const int w = dim / pq_dim;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.0f;
#pragma unroll
    for (int m = 0; m < kMaxM; ++m) {
        if (m < pq_dim) {
            const uint32_t c = code_byte(cw, m);
            const float e = pq_entry<kW>(q + m * w, cent + static_cast<size_t>(c) * dim + m * w, w, keep);
            v[m & 31] = __fadd_rn(v[m & 31], e);
        }
    }
    return butterfly_sum32(v);
}

// Packed codebook for GOFANN_PQ_U8: word (m * 256 + c) * wq + t holds the
// bytes of centroid c's subvector m, dimensions 4t..4t+3 (wq = w / 4).
// Returns false when a centroid value is not an integer in 0..255.
__device__ __forceinline__ bool pack_u8_codebook(const float* __restrict__ cent, int dim, int pq_dim,
                                                 uint32_t* cbw, int tid, int nthreads)
{
    const int w = dim / pq_dim, wq = w / 4;
    const int words = pq_dim * GOFANN_PQ_CENTROIDS * wq;
    bool ok = true;
    for (int i = tid; i < words; i += nthreads) {
        const int t = i % wq, mc = i / wq;
        const int c = mc % GOFANN_PQ_CENTROIDS, m = mc / GOFANN_PQ_CENTROIDS;
        const float* src = cent + static_cast<size_t>(c) * dim + m * w + 4 * t;
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const float v = src[b];
            ok = ok && v >= 0.0f && v <= 255.0f && v == rintf(v);
            word |= (static_cast<uint32_t>(v >= 0.0f && v <= 255.0f ? v : 0.0f) & 0xffu) << (8 * b);
        }
        cbw[i] = word;
    }
    return ok;
}

// GOFANN_PQ_U8 distance: sum over subspaces of |q - c|^2 per byte, as an
// integer (at most 4096 * 255^2 < 2^32; below 2^24 for dim <= 258, where it
// equals the reference's float ADC bit for bit).  qw: query words
// [pq_dim * wq] (shared memory), cbw: packed codebook (shared memory).
template <int kMaxM>
__device__ __forceinline__ float pq_adc_u8(const uint32_t* qw, const uint32_t* cbw, const uint32_t (&cw)[kMaxM / 4],
                                           int pq_dim, int wq)
{
    uint32_t acc = 0;
#pragma unroll
    for (int m = 0; m < kMaxM; ++m) {
        if (m < pq_dim) {
            const uint32_t c = code_byte(cw, m);
            const uint32_t* e = cbw + (m * GOFANN_PQ_CENTROIDS + c) * wq;
            for (int t = 0; t < wq; ++t) {
                const uint32_t d = __vabsdiffu4(qw[m * wq + t], e[t]);
                acc = __dp4a(d, d, acc);
            }
        }
    }
    return __uint2float_rn(acc);
}

// The same for 4-wide subvectors and pq_dim a multiple of 16 (48 at config
// 2), reading the code row 16 bytes at a time inside a loop: one chunk's 16
// subspaces are unrolled, the chunks are not, which keeps the traversal's
// hot loop small (instruction fetch bounds it otherwise); the row's later
// chunks come from L1.
__device__ __forceinline__ float pq_adc_u8_chunked(const uint32_t* qw, const uint32_t* cbw,
                                                   const uint8_t* __restrict__ code, int pq_dim, uint64_t pol)
{
    uint32_t acc = 0, acc2 = 0;
    const uint4* row = reinterpret_cast<const uint4*>(code);
#pragma unroll 1
    for (int q = 0; q < (pq_dim >> 4); ++q) {
        const uint4 x = ldg_u32x4(row + q, pol);
        const uint32_t words[4] = {x.x, x.y, x.z, x.w};
        const uint32_t* cb = cbw + q * 16 * GOFANN_PQ_CENTROIDS;
        const uint32_t* qq = qw + q * 16;
        // two independent accumulators halve the dependent dp4a chain
        // (integer sums: any order gives the same value)
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const uint32_t c0 = (words[j >> 2] >> ((j & 3) * 8)) & 0xffu;
            const uint32_t c1 = (words[j >> 2] >> (((j + 1) & 3) * 8)) & 0xffu;
            const uint32_t d0 = __vabsdiffu4(qq[j], cb[j * GOFANN_PQ_CENTROIDS + c0]);
            const uint32_t d1 = __vabsdiffu4(qq[j + 1], cb[(j + 1) * GOFANN_PQ_CENTROIDS + c1]);
            acc = __dp4a(d0, d0, acc);
            acc2 = __dp4a(d1, d1, acc2);
        }
    }
    return __uint2float_rn(acc + acc2);
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
