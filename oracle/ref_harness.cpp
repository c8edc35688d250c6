// ref_harness.cpp — TEST INFRASTRUCTURE ONLY.
//
// Drives the reference's OWN host-compilable headers (putatio13/GO-FANN,
// included in place from the read-only reference tree at build time, never
// copied) through seeded operation sequences, so that the CPU oracle's
// restatement of those data structures can be pinned against them.  Built by
// oracle/Makefile into oracle/_ref/libgofann_ref.so only where the reference
// tree exists; tests/golden/make_golden.py turns its outputs into committed
// fixtures.
//
// Headers used (include path = <reference>/include and <reference>/src):
//   include/smmh2.h                               symmetric min-max heap
//   include/bin_heap.h                            push_heap / pop_heap
//   search/common/native_visited_hash.cuh         4096-slot visited hash
//   search/common/posting_shortlist_heap.cuh      (dist, id) shortlist heap
//   predicates/gpu_predicate_index.cuh            DNF matches / priority
//   search/rabitq/rabitq_lowfreq_merge.h          route -> original merge
//   data/fp16_l2.h                                fp16 decode and scalar L2
//   index/graph_file_format.h (+ .cpp, compiled)  FDRG graph file writer / loader
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#define __device__
#define __host__
#define __forceinline__ inline

#include "smmh2.h"
#include "bin_heap.h"
#include "search/common/native_visited_hash.cuh"
#include "search/common/posting_shortlist_heap.cuh"
#include "predicates/gpu_predicate_index.cuh"
#include "search/rabitq/rabitq_lowfreq_merge.h"
#include "data/fp16_l2.h"
#include "index/graph_file_format.h"

namespace {

// Same comparison contract as warp_kernel::KernelPair (warp_kernel.cuh:17-26):
// ordering by `first` only.
struct Pair {
    float first;
    uint32_t second;
    bool operator<(const Pair& o) const { return first < o.first; }
    bool operator>(const Pair& o) const { return first > o.first; }
};

}  // namespace

extern "C" {

int ref_seq_smmh(const int* op, const float* key, const uint32_t* payload, int n,
                 float* out_first, uint32_t* out_second, uint32_t* popped)
{
    std::vector<Pair> h(static_cast<size_t>(n) + 2);
    int size = 1, np = 0;
    for (int i = 0; i < n; ++i) {
        if (op[i] == 0) {
            Pair e{key[i], payload[i]};
            smmh2::insert(h.data(), size, e);
        } else if (op[i] == 1 && size > 2) {
            popped[np++] = smmh2::pop_max(h.data(), size).second;
        } else if (op[i] == 2 && size > 1) {
            popped[np++] = smmh2::pop_min(h.data(), size).second;
        }
    }
    for (int i = 0; i < size; ++i) {
        out_first[i] = h[i].first;
        out_second[i] = h[i].second;
    }
    return size;
}

int ref_seq_result_heap(const float* key, const uint32_t* payload, int n, int cap,
                        float* out_first, uint32_t* out_second)
{
    std::vector<Pair> b(static_cast<size_t>(cap) + 2);
    int size = 0;
    for (int i = 0; i < n; ++i) {
        Pair e{key[i], payload[i]};
        if (size < cap) {
            b[size++] = e;
            push_heap(b.data(), b.data() + size);
        } else if (e.first < b[0].first) {
            b[size++] = e;
            push_heap(b.data(), b.data() + size);
            pop_heap(b.data(), b.data() + size);
            --size;
        }
    }
    const int total = size;
    for (int i = 0; i < total; ++i) {
        Pair r = pop_heap(b.data(), b.data() + total - i);
        out_first[i] = r.first;
        out_second[i] = r.second;
    }
    return total;
}

void ref_seq_hash(const uint32_t* values, int n, uint32_t* table, int32_t* found_before)
{
    using namespace go_fann::native_visited_hash;
    for (int i = 0; i < 4096; ++i) table[i] = UINT32_MAX;
    for (int i = 0; i < n; ++i) {
        found_before[i] = test<4096>(table, values[i]) ? 1 : 0;
        add<4096>(table, values[i]);
    }
}

void ref_shortlist(const float* dist, const uint32_t* ids, int n, int k, int sort_out,
                   float* out_d, uint32_t* out_ids)
{
    std::vector<float> d(k, 3.402823466e+38f);
    std::vector<uint32_t> id(k, UINT32_MAX);
    for (int i = 0; i < n; ++i)
        go_fann::posting_shortlist_heap::insert<uint32_t>(dist[i], ids[i], d.data(), id.data(), k);
    if (sort_out) go_fann::posting_shortlist_heap::sort<uint32_t>(d.data(), id.data(), k);
    std::memcpy(out_d, d.data(), sizeof(float) * k);
    std::memcpy(out_ids, id.data(), sizeof(uint32_t) * k);
}

// gpu_predicate::matches over a clause-form View with a sample-major CSR.
void ref_pred_matches(const uint32_t* route_offsets, uint32_t n_routes,
                      const uint32_t* clauses /* [n][4] */, const uint32_t* handles,
                      const uint32_t* ranges /* [n][4] as dimension, mode, lower bits, upper bits */,
                      const float* base_ranges, uint32_t range_stride, const uint32_t* csr_offsets,
                      const uint32_t* csr_labels, uint32_t rows, const uint32_t* query_route,
                      const uint32_t* query_sample, uint32_t n_pairs, uint8_t* out)
{
    using namespace go_fann::gpu_predicate;
    static_assert(sizeof(Clause) == 16, "clause layout");
    static_assert(sizeof(RangeAtom) == 16, "range atom layout");
    View v{};
    v.route_offsets = route_offsets;
    v.route_handles = handles;
    v.clauses = reinterpret_cast<const Clause*>(clauses);
    v.ranges = reinterpret_cast<const RangeAtom*>(ranges);
    v.base_ranges = base_ranges;
    v.range_stride = range_stride;
    v.csr_offsets = csr_offsets;
    v.csr_labels = csr_labels;
    v.rows = rows;
    (void)n_routes;
    for (uint32_t i = 0; i < n_pairs; ++i) out[i] = matches(v, query_route[i], query_sample[i]) ? 1 : 0;
}

void ref_priority(const float* base, const uint8_t* pass, uint32_t n, float penalty, float* out)
{
    for (uint32_t i = 0; i < n; ++i) {
        bool saturated = false;
        out[i] = go_fann::gpu_predicate::priority(base[i], penalty, pass[i] != 0, saturated);
    }
}

// merge_route_results_to_original with the route tables flattened.
int ref_route_merge(const uint32_t* route_to_query, uint32_t n_routes, uint32_t n_queries,
                    const uint32_t* ids, const float* dists, uint32_t width, uint32_t topk,
                    uint32_t* out_ids, float* out_d)
{
    using namespace go_fann::backend_rabitq::lowfreq_merge;
    std::vector<uint32_t> r2q(route_to_query, route_to_query + n_routes);
    std::vector<std::vector<uint32_t>> rr(n_routes);
    std::vector<std::vector<float>> rd(n_routes);
    std::vector<int> steps(n_routes, 1);
    for (uint32_t r = 0; r < n_routes; ++r) {
        rr[r].assign(ids + static_cast<size_t>(r) * width, ids + static_cast<size_t>(r + 1) * width);
        rd[r].assign(dists + static_cast<size_t>(r) * width,
                     dists + static_cast<size_t>(r + 1) * width);
    }
    std::vector<std::vector<uint32_t>> mr;
    std::vector<int> ms;
    std::vector<std::vector<float>> md;
    const auto strategy = merge_route_results_to_original<uint32_t>(r2q, n_queries, rr, rd, steps,
                                                                    topk, mr, ms, &md);
    for (uint32_t q = 0; q < n_queries; ++q)
        for (uint32_t k = 0; k < topk; ++k) {
            out_ids[static_cast<size_t>(q) * topk + k] = k < mr[q].size() ? mr[q][k] : UINT32_MAX;
            out_d[static_cast<size_t>(q) * topk + k] =
                k < md[q].size() ? md[q][k] : 3.402823466e+38f;
        }
    return static_cast<int>(strategy);
}

void ref_fp16_l2(const uint16_t* base, const float* query, uint32_t rows, uint32_t cols, float* out)
{
    for (uint32_t r = 0; r < rows; ++r)
        out[r] = go_fann::fp16_l2::scalar(base + static_cast<size_t>(r) * cols, query, cols);
}

float ref_fp16_decode(uint16_t v) { return go_fann::fp16_l2::decode(v); }

// The reference's FDRG graph file code (src/index/graph_file_format.cpp,
// compiled in place): write rows x degree adjacency with its sequential
// writer, or load a file into a contiguous matrix.  0 = ok, -1 = the
// reference threw (the message is copied into err).
int ref_graph_write(const char* path, const uint32_t* adj, uint64_t rows, uint32_t degree, char* err, int err_len)
{
    try {
        go_fann::graph_file::GraphFileSequentialWriter w(path, rows, degree);
        w.append_rows(adj, rows);
        w.close();
        return 0;
    } catch (const std::exception& e) {
        std::snprintf(err, static_cast<size_t>(err_len), "%s", e.what());
        return -1;
    }
}

int ref_graph_load(const char* path, uint32_t* out, uint64_t capacity, uint64_t* rows, uint64_t* cols, char* err,
                   int err_len)
{
    try {
        const auto m = go_fann::graph_file::load_graph_file_as_contiguous_matrix(path);
        *rows = m.rows;
        *cols = m.cols;
        if (m.data.size() > capacity) return -2;
        std::copy(m.data.begin(), m.data.end(), out);
        return 0;
    } catch (const std::exception& e) {
        std::snprintf(err, static_cast<size_t>(err_len), "%s", e.what());
        return -1;
    }
}

}  // extern "C"
