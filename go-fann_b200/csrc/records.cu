// records.cu — per-row records of the concatenated label graphs.
//
// The reference reaches a candidate's PQ code through row -> sample ->
// code row and its labels through sample -> CSR offsets -> label row
// (GraphMetadata::row_to_sample, pq.codes.bin, SparseLabelMatrix): two
// dependent reads each.  A record stores, per graph row and in row order,
// the sample's code row followed by (sample id, label-row start, label-row
// length, label signature) and, for rows of at most
// GOFANN_RECORD_INLINE_LABELS labels, the labels, so the traversal reads one
// line per candidate.  The records are
// derived data; a traversal gives the same results with or without them.
#include "common.cuh"

namespace gofann {
namespace {

// One thread per 16-byte chunk of a record: code chunks, then the metadata
// chunk, zero padding after.
__global__ void build_records_kernel(gofann_graph g, AttrView at, const uint8_t* __restrict__ codes,
                                     uint32_t pq_dim, uint8_t* __restrict__ out, uint32_t stride, int32_t* status)
{
    const uint32_t chunks = stride / 16;
    const uint32_t meta_chunk = GOFANN_RECORD_META(pq_dim) / 16;
    const uint64_t total = static_cast<uint64_t>(g.total_rows) * chunks;
    for (uint64_t t = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t row = t / chunks;
        const uint32_t c = static_cast<uint32_t>(t - row * chunks);
        const uint32_t sample = g.row_to_sample[row];
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (sample >= at.n_samples) {
            // padding row or corrupt row -> sample entry: an all-zero record
            // (sample 0 with an empty label row) and an error status
            if (c == 0 && status) atomicExch(status, GOFANN_ERR_INVALID);
        } else if (c < meta_chunk) {
            const uint8_t* src = codes + static_cast<uint64_t>(sample) * pq_dim;
            for (uint32_t b = 0; b < 16; ++b) {
                const uint32_t m = c * 16 + b;
                if (m < pq_dim) w[b >> 2] |= static_cast<uint32_t>(src[m]) << ((b & 3) * 8);
            }
        } else if (c == meta_chunk) {
            const uint64_t lo = at.indptr[sample], hi = at.indptr[sample + 1];
            if (hi > 0xffffffffull) {
                if (status) atomicExch(status, GOFANN_ERR_UNSUPPORTED);
            }
            uint32_t sig = 0;
            for (uint64_t k = lo; k < hi; ++k) sig |= GOFANN_LABEL_SIG_BIT(at.indices[k]);
            w[0] = sample;
            w[1] = static_cast<uint32_t>(lo);
            w[2] = static_cast<uint32_t>(hi - lo);
            w[3] = sig;
        } else {
            // inline label row (short rows only)
            const uint64_t lo = at.indptr[sample], hi = at.indptr[sample + 1];
            const uint32_t base = (c - meta_chunk - 1) * 4;
            if (hi - lo <= GOFANN_RECORD_INLINE_LABELS)
                for (uint32_t b = 0; b < 4; ++b)
                    if (base + b < hi - lo) w[b] = at.indices[lo + base + b];
        }
        reinterpret_cast<uint4*>(out + row * stride)[c] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

}  // namespace
}  // namespace gofann

using namespace gofann;

extern "C" {

size_t gofann_row_record_stride(uint32_t pq_dim)
{
    return GOFANN_RECORD_META(pq_dim) + 16u + 4u * GOFANN_RECORD_INLINE_LABELS;
}

int gofann_build_row_records(const gofann_graph* graph, const gofann_attrs* attrs, const gofann_codes* codes,
                             uint8_t* out, int32_t* status, void* stream)
{
    if (!graph || !attrs || !codes || !out) return fail(GOFANN_ERR_INVALID, "build_row_records: null argument");
    if (!graph->row_to_sample || !attrs->label_indptr || !attrs->label_indices || !codes->pq_codes ||
        codes->pq_dim == 0)
        return fail(GOFANN_ERR_INVALID, "build_row_records: row_to_sample, label CSR and PQ codes required");
    if ((reinterpret_cast<uintptr_t>(out) & 15) != 0)
        return fail(GOFANN_ERR_INVALID, "build_row_records: output must be 16-byte aligned");
    if (graph->total_rows == 0) return GOFANN_OK;
    AttrView at{};
    at.indptr = attrs->label_indptr;
    at.indices = attrs->label_indices;
    at.n_samples = attrs->n_samples;
    const uint32_t stride = static_cast<uint32_t>(gofann_row_record_stride(codes->pq_dim));
    const uint64_t work = static_cast<uint64_t>(graph->total_rows) * (stride / 16);
    const int threads = 256;
    const uint64_t want = (work + threads - 1) / threads;
    const int sms = sm_count() > 0 ? sm_count() : 148;
    const unsigned blocks = static_cast<unsigned>(want < static_cast<uint64_t>(sms) * 32 ? want : sms * 32);
    build_records_kernel<<<blocks, threads, 0, as_stream(stream)>>>(*graph, at, codes->pq_codes, codes->pq_dim, out,
                                                                    stride, status);
    GOFANN_CHECK_LAUNCH("build_records_kernel");
    return GOFANN_OK;
}

}  // extern "C"
