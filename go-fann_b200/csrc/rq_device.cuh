// rq_device.cuh — device-side 1-bit RaBitQ estimator.
//
// The integer inner product sum_{d: bit(d)} q8[d] is computed from the 8 bit
// planes of the two's-complement query bytes, q8[d] = sum_{b<7} 2^b bit_b(d)
// - 128 bit_7(d):  ip = sum_{b<7} 2^b popc(code & plane_b) - 128
// popc(code & plane_7).  Integer sums are exact, so this equals the
// reference's dp4a nibble-mask form (backend_rabitq.cu:3070-3098) bit for
// bit, with one popc per plane per 32 dimensions instead of 8 dp4a + 8 table
// loads.  Code bit layout: dimension d is bit 31-(d%32) of little-endian
// word d/32.
#pragma once

#include "common.cuh"

namespace gofann {

constexpr int kMaxRqWords = 4096 / 32;  // padded_dim <= 4096

// Builds the 8 bit planes [8][words] of one query into shared memory.
// Cooperative over `nthreads` threads starting at `tid`.
__device__ __forceinline__ void rq_build_planes(const int8_t* __restrict__ q8, int padded_dim,
                                                uint32_t* planes, int tid, int nthreads)
{
    const int words = padded_dim / 32;
    for (int w = tid; w < words; w += nthreads) {
        uint32_t p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int k = 0; k < 32; ++k) {
            const uint32_t u = static_cast<uint8_t>(q8[w * 32 + k]);
#pragma unroll
            for (int b = 0; b < 8; ++b) p[b] |= ((u >> b) & 1u) << (31 - k);
        }
#pragma unroll
        for (int b = 0; b < 8; ++b) planes[b * words + w] = p[b];
    }
}

// Inner product of one code word with the planes p[0..7] of its 32 dimensions.
__device__ __forceinline__ int32_t rq_word_ip_planes(uint32_t code_w, uint32_t p0, uint32_t p1, uint32_t p2,
                                                     uint32_t p3, uint32_t p4, uint32_t p5, uint32_t p6,
                                                     uint32_t p7)
{
    int32_t acc = __popc(code_w & p0);
    acc += __popc(code_w & p1) << 1;
    acc += __popc(code_w & p2) << 2;
    acc += __popc(code_w & p3) << 3;
    acc += __popc(code_w & p4) << 4;
    acc += __popc(code_w & p5) << 5;
    acc += __popc(code_w & p6) << 6;
    return acc - (__popc(code_w & p7) << 7);
}

// Carry-save adders on 32 bit lanes: x + y + z = s + 2 c (full adder), x + y
// = s + 2 c (half adder), every bit position independently.
__device__ __forceinline__ void csa_full(uint32_t x, uint32_t y, uint32_t z, uint32_t& s, uint32_t& c)
{
    s = x ^ y ^ z;
    c = (x & y) | (z & (x ^ y));
}
__device__ __forceinline__ void csa_half(uint32_t x, uint32_t y, uint32_t& s, uint32_t& c)
{
    s = x ^ y;
    c = x & y;
}

// Inner product of 4 code words c[0..3] with their planes p[b][0..3]:
// sum_{b<7} 2^b sum_j popc(c_j & p_bj) - 128 sum_j popc(c_j & p_7j).  The
// 28 masked words of weights 1..64 are reduced column by column with
// carry-save adders (a column's carries join the next column) to one word
// per weight 1..256, and the 4 words of weight -128 to one word per weight
// 128..512: 12 popc instead of 32 (popc issues at a quarter of the integer
// logic rate).  Exact integer arithmetic: the same value as
// rq_word_ip_planes summed over the 4 words.
__device__ __forceinline__ int32_t rq_ip4_csa(const uint32_t (&c)[4], const uint32_t (&p)[8][4])
{
    uint32_t col[9];
    uint32_t k0, k1, k2;  // carries into the current column
    {   // weight 1: 4 words -> 1, carries 2
        uint32_t s;
        csa_full(c[0] & p[0][0], c[1] & p[0][1], c[2] & p[0][2], s, k0);
        csa_half(s, c[3] & p[0][3], col[0], k1);
    }
    {   // weight 2: 4 words + 2 carries -> 1, carries 3
        uint32_t s, s2, n0, n1, n2;
        csa_full(k0, k1, c[0] & p[1][0], s, n0);
        csa_full(c[1] & p[1][1], c[2] & p[1][2], c[3] & p[1][3], s2, n1);
        csa_half(s, s2, col[1], n2);
        k0 = n0; k1 = n1; k2 = n2;
    }
#pragma unroll
    for (int b = 2; b < 7; ++b) {  // weights 4..64: 4 words + 3 carries -> 1, carries 3
        uint32_t s, s2, n0, n1, n2;
        csa_full(k0, k1, k2, s, n0);
        csa_full(c[0] & p[b][0], c[1] & p[b][1], c[2] & p[b][2], s2, n1);
        csa_full(s, s2, c[3] & p[b][3], col[b], n2);
        k0 = n0; k1 = n1; k2 = n2;
    }
    csa_full(k0, k1, k2, col[7], col[8]);  // weights 128 and 256
    uint32_t ng0, ng1, ng2;                // weight -128 words -> weights 128, 256, 512
    {
        uint32_t s, e0, e1;
        csa_full(c[0] & p[7][0], c[1] & p[7][1], c[2] & p[7][2], s, e0);
        csa_half(s, c[3] & p[7][3], ng0, e1);
        csa_half(e0, e1, ng1, ng2);
    }
    int32_t acc = 0;
#pragma unroll
    for (int b = 0; b < 9; ++b) acc += __popc(col[b]) << b;
    return acc - ((__popc(ng0) + (__popc(ng1) << 1) + (__popc(ng2) << 2)) << 7);
}

__device__ __forceinline__ int32_t rq_word_ip(uint32_t code_w, const uint32_t* planes, int words, int w)
{
    return rq_word_ip_planes(code_w, planes[w], planes[words + w], planes[2 * words + w], planes[3 * words + w],
                             planes[4 * words + w], planes[5 * words + w], planes[6 * words + w],
                             planes[7 * words + w]);
}

// Whole-code inner product by one thread (codes 16-byte aligned when
// code_bytes % 16 == 0).
__device__ __forceinline__ int32_t rq_ip_thread(const uint8_t* __restrict__ code, const uint32_t* planes,
                                                int words)
{
    int32_t acc = 0;
    if ((words & 3) == 0 && (reinterpret_cast<uintptr_t>(code) & 15) == 0) {
        const uint4* p = reinterpret_cast<const uint4*>(code);
        for (int i = 0; i < words / 4; ++i) {
            const uint4 x = __ldg(p + i);
            acc += rq_word_ip(x.x, planes, words, 4 * i + 0);
            acc += rq_word_ip(x.y, planes, words, 4 * i + 1);
            acc += rq_word_ip(x.z, planes, words, 4 * i + 2);
            acc += rq_word_ip(x.w, planes, words, 4 * i + 3);
        }
    } else {
        const uint32_t* p = reinterpret_cast<const uint32_t*>(code);
        for (int i = 0; i < words; ++i) acc += rq_word_ip(__ldg(p + i), planes, words, i);
    }
    return acc;
}

// Combine of score_rabitq_code_device (backend_rabitq.cu:3185-3192), pinned
// as fma(f_rescale, fma(float(ip), scale, k1xsumq), f_add + gdist).
__device__ __forceinline__ float rq_combine(int32_t ip, float scale, float k1, float f_add,
                                            float f_rescale, float gdist)
{
    const float t = __fmaf_rn(static_cast<float>(ip), scale, k1);
    return __fmaf_rn(f_rescale, t, __fadd_rn(f_add, gdist));
}

struct RqQueryView {
    const uint32_t* planes;  // [8][words] (shared memory)
    float scale, k1;
    const float* gdist;      // [num_anchors] of this query row
};

__device__ __forceinline__ float rq_estimate(const gofann_codes& c, const RqQueryView& q, uint32_t sample)
{
    const int words = static_cast<int>(c.padded_dim / 32);
    const int32_t ip = rq_ip_thread(c.rq_codes + static_cast<size_t>(sample) * (c.padded_dim / 8), q.planes,
                                    words);
    const float f_add = __ldg(c.rq_factors + static_cast<size_t>(sample) * 3);
    const float f_rescale = __ldg(c.rq_factors + static_cast<size_t>(sample) * 3 + 1);
    const uint32_t anchor = __ldg(c.rq_anchor_ids + sample);
    return rq_combine(ip, q.scale, q.k1, f_add, f_rescale, __ldg(q.gdist + anchor));
}

}  // namespace gofann
