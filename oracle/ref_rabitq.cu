// ref_rabitq.cu — TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's RaBitQ search backend (putatio13/GO-FANN
// src/search/rabitq/backend_rabitq.cu) in place from the read-only reference
// tree -- nothing is copied -- and exposes one C entry point that runs its
// 1-bit estimator, score_rabitq_code_device<kUseInt8Score = true>
// (backend_rabitq.cu:3100-3200), on (query row, point) pairs: one warp per
// pair, lane = subtid, the int8 query and its scale, k1xsumq and the centroid
// distances of the prepared state, exactly the arguments its traversal and
// posting scans pass for a 1-bit index (bits_per_dim 1: no long codes, no
// extra factors).  The GDRCopy calls of the file's host half are declared by
// oracle/ref_stub/ and defined below as failing stubs that nothing calls.
#include "type_def.h"
#undef dist_t
#undef pq_value_t
typedef float gofann_ref_float;
#define dist_t gofann_ref_float
#define pq_value_t gofann_ref_float
#include "search/rabitq/backend_rabitq.cu"

extern "C" {
gdr_t gdr_open(void) { return nullptr; }
int gdr_close(gdr_t) { return -1; }
int gdr_pin_buffer(gdr_t, unsigned long, size_t, uint64_t, uint32_t, gdr_mh_t*) { return -1; }
int gdr_unpin_buffer(gdr_t, gdr_mh_t) { return -1; }
int gdr_map(gdr_t, gdr_mh_t, void**, size_t) { return -1; }
int gdr_unmap(gdr_t, gdr_mh_t, void*, size_t) { return -1; }
}

namespace gofann_ref_rq {

__global__ void ref_rq_score_pairs(const uint32_t* anchor_ids, const uint8_t* codes, const float* factors,
                                   const float* k1xsumq, const float* gdist, const int8_t* q8, const float* scales,
                                   const uint32_t* pair_row, const uint32_t* pair_point, uint32_t n_pairs,
                                   uint32_t num_anchors, uint32_t padded_dim, float* out)
{
    const uint32_t p = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = static_cast<int>(threadIdx.x & 31u);
    if (p >= n_pairs) return;
    const float d = go_fann::backend_rabitq::score_rabitq_code_device<true>(
        anchor_ids, codes, nullptr, factors, nullptr, nullptr, nullptr, k1xsumq, nullptr, gdist, pair_row[p],
        pair_point[p], num_anchors, padded_dim, padded_dim / 8u, 0u, 1u, lane, q8, scales);
    if (lane == 0) out[p] = d;
}

}  // namespace gofann_ref_rq

extern "C" {

// Device pointers; 0 = launched, -2 = launch error.
__attribute__((visibility("default"))) int gofann_ref_rq_score(const uint32_t* anchor_ids, const uint8_t* codes,
                                                               const float* factors, const float* k1xsumq,
                                                               const float* gdist, const int8_t* q8,
                                                               const float* scales, const uint32_t* pair_row,
                                                               const uint32_t* pair_point, uint32_t n_pairs,
                                                               uint32_t num_anchors, uint32_t padded_dim, float* out)
{
    if (n_pairs == 0) return 0;
    const unsigned blocks = (n_pairs + 3u) / 4u;
    gofann_ref_rq::ref_rq_score_pairs<<<blocks, 128>>>(anchor_ids, codes, factors, k1xsumq, gdist, q8, scales,
                                                       pair_row, pair_point, n_pairs, num_anchors, padded_dim, out);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // extern "C"
