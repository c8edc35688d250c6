// exact_device.cuh — exact L2 distances between a query and full base
// vectors resident in HBM, in the arithmetic of the reference's Full-GPU
// backend (l2_distance_device, src/search/full_gpu/backend_full_gpu.cu:
// 1106-1190), for the exact-distance traversal and posting scans.
//
//  * u8: the reference sums |x|^2 + |q|^2 - 2 x.q with dp4a in uint32, which
//    is the integer sum of squared byte differences; here that sum is taken
//    directly (per-byte absolute difference, then a dot product of the packed
//    differences with themselves) and converted to float the same way.
//  * f32: lane l sums (x_d - q_d)^2 over d = l, l+32, ... with one fma per
//    term (nvcc contracts `partial += diff * diff`), then lane 0 receives the
//    shfl_down tree 16, 8, 4, 2, 1.
//  * f16 (even dim): lane l sums over the half2 pairs p = l, l+32, ...
//    partial + (dx*dx + dy*dy) with the pair term contracted as
//    fma(dx, dx, dy*dy); odd dims take the f32 form on converted halves.
// The warp form computes one candidate with 32 lanes exactly as the
// reference does; the thread form replays the same 32 partials and the tree
// inside one thread (lane 0's tree value equals the xor butterfly's).
#pragma once

#include "common.cuh"

namespace gofann {

__device__ __forceinline__ uint32_t sq_absdiff_u8x4(uint32_t a, uint32_t b, uint32_t acc)
{
    const uint32_t d = __vabsdiffu4(a, b);
    return __dp4a(d, d, acc);
}

// Squared L2 of a u8 row (16-byte aligned, n16 16-byte chunks) against the
// query's chunks q16 (shared memory), one thread.
__device__ __forceinline__ uint32_t l2_u8_thread(const uint8_t* row, const uint4* q16, int n16, uint64_t pol)
{
    const uint4* r = reinterpret_cast<const uint4*>(row);
    uint32_t acc = 0;
    int c = 0;
    for (; c + 8 <= n16; c += 8) {
        uint4 x[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) x[u] = ldg_u32x4(r + c + u, pol);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const uint4 y = q16[c + u];
            acc = sq_absdiff_u8x4(x[u].x, y.x, acc);
            acc = sq_absdiff_u8x4(x[u].y, y.y, acc);
            acc = sq_absdiff_u8x4(x[u].z, y.z, acc);
            acc = sq_absdiff_u8x4(x[u].w, y.w, acc);
        }
    }
    if (c + 4 <= n16) {
        uint4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = ldg_u32x4(r + c + u, pol);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint4 y = q16[c + u];
            acc = sq_absdiff_u8x4(x[u].x, y.x, acc);
            acc = sq_absdiff_u8x4(x[u].y, y.y, acc);
            acc = sq_absdiff_u8x4(x[u].z, y.z, acc);
            acc = sq_absdiff_u8x4(x[u].w, y.w, acc);
        }
        c += 4;
    }
    for (; c < n16; ++c) {
        const uint4 x = ldg_u32x4(r + c, pol), y = q16[c];
        acc = sq_absdiff_u8x4(x.x, y.x, acc);
        acc = sq_absdiff_u8x4(x.y, y.y, acc);
        acc = sq_absdiff_u8x4(x.z, y.z, acc);
        acc = sq_absdiff_u8x4(x.w, y.w, acc);
    }
    return acc;
}

// One term of the f16 pair loop: dx*dx + dy*dy as nvcc contracts it.
__device__ __forceinline__ float f16_pair_term(float dx, float dy)
{
    return __fmaf_rn(dx, dx, __fmul_rn(dy, dy));
}

// Lane 0's value of the shfl_down tree 16..1, broadcast to every lane.
__device__ __forceinline__ float warp_tree_sum(float v)
{
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_down_sync(kFull, v, off));
    return __shfl_sync(kFull, v, 0);
}

// Exact L2 of kN rows at once (rows[u] may be null: skipped) against the
// query q (shared memory), the reference's warp order; every lane returns
// the distances.  Rows are read with loads interleaved across the kN rows.
template <int kDtype, int kN>
__device__ __forceinline__ void l2_float_warp(const void* const (&rows)[kN], const void* q, int dim, int lane,
                                              uint64_t pol, float (&out)[kN])
{
    float part[kN];
#pragma unroll
    for (int u = 0; u < kN; ++u) part[u] = 0.0f;
    if constexpr (kDtype == GOFANN_DTYPE_F32) {
        const float* qf = static_cast<const float*>(q);
        for (int d = lane; d < dim; d += kWarp) {
            const float qd = qf[d];
            float x[kN];
#pragma unroll
            for (int u = 0; u < kN; ++u)
                x[u] = rows[u] ? ldg_f32(static_cast<const float*>(rows[u]) + d, pol) : qd;
#pragma unroll
            for (int u = 0; u < kN; ++u) {
                const float diff = __fsub_rn(x[u], qd);
                part[u] = __fmaf_rn(diff, diff, part[u]);
            }
        }
    } else {
        const __half* qh = static_cast<const __half*>(q);
        if ((dim & 1) == 0) {
            const int dim2 = dim / 2;
            const __half2* q2 = reinterpret_cast<const __half2*>(qh);
            for (int d = lane; d < dim2; d += kWarp) {
                const float2 qv = __half22float2(q2[d]);
                uint32_t x[kN];
#pragma unroll
                for (int u = 0; u < kN; ++u)
                    x[u] = rows[u] ? ldg_u32(static_cast<const uint32_t*>(rows[u]) + d, pol) : 0u;
#pragma unroll
                for (int u = 0; u < kN; ++u) {
                    __half2 h;
                    memcpy(&h, &x[u], 4);
                    const float2 b = __half22float2(h);
                    const float dx = __fsub_rn(b.x, qv.x);
                    const float dy = __fsub_rn(b.y, qv.y);
                    part[u] = __fadd_rn(part[u], f16_pair_term(dx, dy));
                }
            }
        } else {
            for (int d = lane; d < dim; d += kWarp) {
                const float qd = __half2float(qh[d]);
#pragma unroll
                for (int u = 0; u < kN; ++u) {
                    const float b = rows[u] ? __half2float(static_cast<const __half*>(rows[u])[d]) : qd;
                    const float diff = __fsub_rn(b, qd);
                    part[u] = __fmaf_rn(diff, diff, part[u]);
                }
            }
        }
    }
#pragma unroll
    for (int u = 0; u < kN; ++u) out[u] = warp_tree_sum(part[u]);
}

// The same distance computed by one thread: the 32 lane partials, then the
// tree (butterfly_sum32 gives lane 0's tree value).
template <int kDtype>
__device__ __forceinline__ float l2_float_thread(const void* row, const void* q, int dim)
{
    float v[32];
#pragma unroll
    for (int l = 0; l < 32; ++l) v[l] = 0.0f;
    if constexpr (kDtype == GOFANN_DTYPE_F32) {
        const float* x = static_cast<const float*>(row);
        const float* qf = static_cast<const float*>(q);
        for (int d0 = 0; d0 < dim; d0 += kWarp) {
#pragma unroll
            for (int l = 0; l < 32; ++l) {
                const int d = d0 + l;
                if (d < dim) {
                    const float diff = __fsub_rn(__ldg(x + d), qf[d]);
                    v[l] = __fmaf_rn(diff, diff, v[l]);
                }
            }
        }
    } else {
        const __half* x = static_cast<const __half*>(row);
        const __half* qh = static_cast<const __half*>(q);
        if ((dim & 1) == 0) {
            const int dim2 = dim / 2;
            const uint32_t* x2 = reinterpret_cast<const uint32_t*>(x);
            const __half2* q2 = reinterpret_cast<const __half2*>(qh);
            for (int p0 = 0; p0 < dim2; p0 += kWarp) {
#pragma unroll
                for (int l = 0; l < 32; ++l) {
                    const int p = p0 + l;
                    if (p < dim2) {
                        const uint32_t w = __ldg(x2 + p);
                        __half2 h;
                        memcpy(&h, &w, 4);
                        const float2 b = __half22float2(h);
                        const float2 qv = __half22float2(q2[p]);
                        v[l] = __fadd_rn(v[l], f16_pair_term(__fsub_rn(b.x, qv.x), __fsub_rn(b.y, qv.y)));
                    }
                }
            }
        } else {
            for (int d0 = 0; d0 < dim; d0 += kWarp) {
#pragma unroll
                for (int l = 0; l < 32; ++l) {
                    const int d = d0 + l;
                    if (d < dim) {
                        const float diff = __fsub_rn(__half2float(x[d]), __half2float(qh[d]));
                        v[l] = __fmaf_rn(diff, diff, v[l]);
                    }
                }
            }
        }
    }
    return butterfly_sum32(v);
}

}  // namespace gofann
