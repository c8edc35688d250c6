// ref_kernels.cu — TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's PQ search backend (putatio13/GO-FANN
// src/search/pq/backend_pq.cu) in place from the read-only reference tree --
// nothing is copied -- and exposes one C entry point that launches its
// device-resident traversal kernel,
//   native_warp_independent_search_kernel_impl<QS, PD, /*request ring*/ false,
//                                              /*device resident*/ true, bias>
// (backend_pq.cu:5015-5199, body run_pq_search_one_block :3988-5013),
// exactly as the reference's host driver launches it (backend_pq.cu:
// 10303-10378): one 32-thread block per route, dynamic shared memory
// native_pq_workspace_shared_bytes(queue_size, result_width, bias).  The
// kernel builds the route's PQ table itself (computePQTable, :1999-2022) into
// pq_table, so the table, the traversal ids, distances, step counts and the
// expansion trace can all be compared with the CPU oracle and with the
// library's own kernel on the same seeded inputs.
//
// The device-resident branch reads only device arrays: every mailbox /
// GDRCopy / request-ring access and every wait on a host flag sits under
// `if constexpr (!kDeviceResident)` or `kUseRequestRing` (backend_pq.cu:
// 4107-4126, 4312-4375, 4456-4492, 4700, 4730, 4980-5011), so this harness
// passes null for those pointers and defines the GDRCopy calls (declared in
// oracle/ref_stub/gdrapi.h, needed only to compile the host half of the
// file) as failing stubs that nothing calls.
//
// Two build adjustments, both about the reference's own headers and not its
// arithmetic: include/type_def.h defines `dist_t` and `pq_value_t` as the
// macro `_Float32`, which include/config1B.h then re-declares with
// `typedef float dist_t`; with GCC 13 `_Float32` is a built-in type and that
// typedef does not compile, so both macros are redirected to a float typedef
// before the backend is included (dist_t is float either way).
#include "type_def.h"
#undef dist_t
#undef pq_value_t
typedef float gofann_ref_float;
#define dist_t gofann_ref_float
#define pq_value_t gofann_ref_float
#include "search/pq/backend_pq.cu"

extern "C" {
gdr_t gdr_open(void) { return nullptr; }
int gdr_close(gdr_t) { return -1; }
int gdr_pin_buffer(gdr_t, unsigned long, size_t, uint64_t, uint32_t, gdr_mh_t*) { return -1; }
int gdr_unpin_buffer(gdr_t, gdr_mh_t) { return -1; }
int gdr_map(gdr_t, gdr_mh_t, void**, size_t) { return -1; }
int gdr_unmap(gdr_t, gdr_mh_t, void*, size_t) { return -1; }
}

// Arguments of one reference launch: device pointers and scalars.  Route r
// searches query row r (the reference indexes its queries, tables and
// outputs by route).
struct gofann_ref_pq_args {
    const uint8_t* codes;            // [n_samples][pq_dim]
    const float* centroids;          // [256][dim]
    const uint8_t* queries;          // [n_routes][dim]
    const uint32_t* adjacency;       // [total_rows][degree]
    const uint32_t* row_to_sample;   // [total_rows]
    const uint32_t* label_offset;    // [groups]
    const uint32_t* zero_groups;     // [groups] zeros (no static prefetch)
    const uint64_t* data_indptr;     // [n_samples + 1]
    const uint32_t* data_indptr32;   // [n_samples + 1] (gpu_predicate CSR view)
    const uint32_t* data_indices;    // [nnz]
    const uint32_t* group_id;        // [n_routes]
    const uint32_t* start_local;     // [n_routes]
    const uint64_t* filter_bits;     // [n_routes]
    const uint64_t* qlabel_indptr;   // [n_routes + 1]
    const uint32_t* qlabel_indices;
    const uint32_t* primary_label;   // [n_routes]
    const uint32_t* pred_offsets;    // [n_routes + 1] into clauses, or null = no predicate
    const void* clauses;             // gpu_predicate::Clause [..]
    const uint32_t* pred_handles;
    const uint8_t* pred_enabled;     // [n_routes]
    uint64_t* out_ids;               // [n_routes][result_width]
    float* out_dists;                // [n_routes][result_width]
    float* pq_table;                 // [n_routes][pd_capacity][256]
    uint32_t* hash;                  // [n_routes][4096]
    float* time_per_block;           // [n_routes][6] (slot 4 = step count)
    float* datadist;                 // scratch the kernel receives (unused when resident)
    uint32_t* trace_rows;            // [n_routes][trace_width] or null
    uint32_t* trace_slots;           // [n_routes] = 0..n-1
    uint32_t* trace_counters;        // [n_routes][3] zeros
    uint32_t trace_width;
    uint32_t n_samples, dim, pq_dim, degree, n_routes;
    int32_t queue_size, finish_limit, early_stop_mode, max_steps, stop_width, result_width;
    int32_t predicate_bias, full_label_check, pending_base_stop;
    float alpha;
};

namespace {

template <int QS, int PD, bool kBias>
int launch_ref(const gofann_ref_pq_args& a)
{
    using namespace go_fann::backend_pq;
    go_fann::gpu_predicate::View pv{};
    if (a.pred_offsets) {
        pv.route_offsets = a.pred_offsets;
        pv.route_handles = a.pred_handles;
        pv.rows = a.n_samples;
        pv.alpha = a.alpha;
        pv.clauses = static_cast<const go_fann::gpu_predicate::Clause*>(a.clauses);
        pv.route_enabled = a.pred_enabled;
        pv.pending_base_stop = a.pending_base_stop != 0;
        pv.csr_offsets = a.data_indptr32;
        pv.csr_labels = a.data_indices;
    }
    go_fann::expansion_trace::View ev{};
    if (a.trace_rows) {
        ev.rows = a.trace_rows;
        ev.route_slots = a.trace_slots;
        ev.counters = reinterpret_cast<go_fann::expansion_trace::Counters*>(a.trace_counters);
        ev.capacity = a.trace_width;
    }
    const size_t smem = native_pq_workspace_shared_bytes(static_cast<uint32_t>(a.queue_size),
                                                         static_cast<uint32_t>(a.result_width), kBias);
    native_warp_independent_search_kernel_impl<QS, PD, false, true, kBias>
        <<<static_cast<int>(a.n_routes), kNativeResidentThreadInBlock, smem>>>(
            a.codes, nullptr, const_cast<uint8_t*>(a.queries), reinterpret_cast<idx_t*>(a.out_ids), a.out_dists,
            a.centroids, a.pq_table, a.datadist, a.hash, static_cast<int>(a.n_routes), a.time_per_block, nullptr,
            nullptr, a.adjacency, a.degree, a.data_indptr, a.data_indices, a.qlabel_indptr, a.qlabel_indices,
            a.primary_label, a.full_label_check, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0u, nullptr,
            nullptr, a.zero_groups, a.zero_groups, a.group_id, a.start_local, a.start_local, a.row_to_sample,
            a.label_offset, nullptr, a.filter_bits, nullptr, nullptr, nullptr, nullptr, 0u,
            static_cast<int>(a.dim), static_cast<int>(a.pq_dim), 0, 0, a.queue_size, a.finish_limit,
            a.early_stop_mode, a.max_steps, a.stop_width, a.result_width, 0u, 0u, 0u, 0u, 0u, 0u,
            /*use_sample_id_payload*/ 0, /*use_implicit_filter_mask*/ 1, /*enable_true_distance_rerank*/ 0,
            1.0f, 1.0f, 0, pv, ev);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        std::fprintf(stderr, "reference PQ kernel launch: %s\n", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}

template <int PD, bool kBias>
int by_queue(const gofann_ref_pq_args& a)
{
    switch (go_fann::backend_pq::specialized_queue_capacity(a.queue_size)) {
    case 64: return launch_ref<64, PD, kBias>(a);
    case 128: return launch_ref<128, PD, kBias>(a);
    case 256: return launch_ref<256, PD, kBias>(a);
    case 512: return launch_ref<512, PD, kBias>(a);
    default: return -1;
    }
}

// The reference's cooperative pickup (backend_pq.cu:844-893), instantiated
// for its biased frontier entries, on crafted frontiers: one warp per
// frontier of `stride` entries (index 0 unused, heap size sizes[c]); entry
// i carries payload i (bit 31 = used), so the picked index is read back.
__global__ void ref_pickup_cases(go_fann::gpu_predicate::BiasedPair* frontiers, const int* sizes, int stride,
                                 int* picked)
{
    go_fann::gpu_predicate::BiasedPair* f = frontiers + static_cast<size_t>(blockIdx.x) * stride;
    go_fann::gpu_predicate::BiasedPair out;
    const bool found = go_fann::backend_pq::pickup_next_unused_from_native_frontier<true>(
        f, sizes[blockIdx.x], out, static_cast<int>(threadIdx.x));
    if (threadIdx.x == 0) picked[blockIdx.x] = found ? static_cast<int>(out.second & 0x7fffffffu) : -1;
}

// The reference's result heap (include/bin_heap.h push_heap / pop_heap on
// ResultPair, as run_pq_search_one_block uses it, backend_pq.cu:4619-4628
// and 4968-4982): one thread per sequence; keys[i] are offered in order to a
// heap of capacity cap, then the heap is emptied by pop_heap into ascending
// output slots.
__global__ void ref_result_heap_cases(const float* keys, const uint32_t* payloads, int n, int cap,
                                      float* out_first, uint32_t* out_second)
{
    using go_fann::backend_pq::ResultPair;
    extern __shared__ __align__(8) unsigned char heap_raw[];
    ResultPair* h = reinterpret_cast<ResultPair*>(heap_raw);
    const size_t c = blockIdx.x;
    if (threadIdx.x != 0) return;
    int size = 0;
    for (int i = 0; i < n; ++i) {
        ResultPair e;
        e.first = keys[c * n + i];
        e.second = payloads[c * n + i];
        if (size < cap) {
            h[size++] = e;
            push_heap(h, h + size);
        } else if (e.first < h[0].first) {
            h[size++] = e;
            push_heap(h, h + size);
            pop_heap(h, h + size);
            --size;
        }
    }
    for (int i = 0; i < cap; ++i) {
        out_first[c * cap + i] = FLT_MAX;
        out_second[c * cap + i] = UINT32_MAX;
    }
    for (int i = 0; i < size; ++i) {
        ResultPair r = pop_heap(h, h + size - i);
        out_first[c * cap + size - 1 - i] = r.first;
        out_second[c * cap + size - 1 - i] = r.second;
    }
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int gofann_ref_pickup_cases(void* frontiers, const int* sizes, int n_cases,
                                                                   int stride, int* picked)
{
    if (n_cases <= 0) return 0;
    ref_pickup_cases<<<n_cases, 32>>>(static_cast<go_fann::gpu_predicate::BiasedPair*>(frontiers), sizes, stride,
                                      picked);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

__attribute__((visibility("default"))) int gofann_ref_result_heap_cases(const float* keys, const uint32_t* payloads,
                                                                        int n_cases, int n, int cap,
                                                                        float* out_first, uint32_t* out_second)
{
    if (n_cases <= 0) return 0;
    if (cap < 1 || cap > 1024) return -1;
    ref_result_heap_cases<<<n_cases, 32, static_cast<size_t>(cap + 1) * 8>>>(keys, payloads, n, cap, out_first,
                                                                             out_second);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Launches the reference's device-resident PQ traversal on the current
// stream of the current device (legacy default stream); returns 0, -1 for a
// shape the reference does not compile (pq_dim other than 16 or 64, queue
// above 512, dim above 192), -2 for a launch error.
__attribute__((visibility("default"))) int gofann_ref_pq_search(const gofann_ref_pq_args* a)
{
    if (!a || a->queue_size < 2 || a->queue_size > 512 || a->dim > 192 || a->dim == 0 ||
        a->result_width < 1 || a->stop_width < 1 || a->stop_width > 10 || a->degree > 64)
        return -1;
    const bool bias = a->predicate_bias != 0;
    if (a->pq_dim == 16) return bias ? by_queue<16, true>(*a) : by_queue<16, false>(*a);
    if (a->pq_dim == 64) return bias ? by_queue<64, true>(*a) : by_queue<64, false>(*a);
    return -1;
}

__attribute__((visibility("default"))) size_t gofann_ref_pq_args_size(void) { return sizeof(gofann_ref_pq_args); }

}  // extern "C"
