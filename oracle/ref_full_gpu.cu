// ref_full_gpu.cu — TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's Full-GPU search backend (putatio13/GO-FANN
// src/search/full_gpu/backend_full_gpu.cu) in place from the read-only
// reference tree -- nothing is copied -- and exposes C entry points that
// launch its exact-distance kernels exactly as its host driver does
// (launch_search_kernels_for_routes, backend_full_gpu.cu:2955-3165):
//   * full_gpu_highfreq_kernel<kQueueSize, T, false> (:2044-2122, body
//     run_full_gpu_highfreq_route :1682-2043): one 128-thread block per
//     graph route, dim * sizeof(T) bytes of dynamic shared memory;
//   * full_gpu_lowfreq_kernel<T> (:2124-2260): one 32-thread block per
//     posting route;
//   * pickup_next_unused_from_pool_block (:1536-1596) on crafted frontiers.
// T is uint8_t, float or __half.  The kernels read only device arrays; the
// GDRCopy calls of the file's host half are declared by oracle/ref_stub/
// and defined below as failing stubs that nothing calls.
#include "type_def.h"
#undef dist_t
#undef pq_value_t
typedef float gofann_ref_float;
#define dist_t gofann_ref_float
#define pq_value_t gofann_ref_float
#include "search/full_gpu/backend_full_gpu.cu"

extern "C" {
gdr_t gdr_open(void) { return nullptr; }
int gdr_close(gdr_t) { return -1; }
int gdr_pin_buffer(gdr_t, unsigned long, size_t, uint64_t, uint32_t, gdr_mh_t*) { return -1; }
int gdr_unpin_buffer(gdr_t, gdr_mh_t) { return -1; }
int gdr_map(gdr_t, gdr_mh_t, void**, size_t) { return -1; }
int gdr_unmap(gdr_t, gdr_mh_t, void*, size_t) { return -1; }
}

// Device pointers and scalars of one launch, named after the kernels'
// parameters.  dtype: 0 = uint8, 1 = float, 2 = half.
struct gofann_ref_full_args {
    const void* base;
    const void* queries;
    const uint32_t* graph;
    const uint32_t* active_ids;          // [n_routes] = 0..n-1
    const uint32_t* query_vector_ids;    // route -> query row
    const uint32_t* group_ids;
    const uint32_t* start_local;
    const uint32_t* label_size;
    const uint32_t* label_offset;
    const uint32_t* row_to_sample;
    const uint64_t* row_filter_mask;     // graph rows (highfreq) or posting entries (lowfreq)
    const uint64_t* filter_bits;
    const uint8_t* filter_modes;
    const uint32_t* single_extra;
    const uint32_t* active_range_counts;
    const uint32_t* qlabel_indptr;       // u32 [n_routes + 1]
    const uint32_t* qlabel_indices;
    const uint32_t* sample_indptr;       // u32 [n_samples + 1]
    const uint32_t* sample_indices;
    const uint8_t* range_modes;
    const float* range_lower;
    const float* range_upper;
    const float* base_ranges;
    const uint32_t* low_sample_ids;      // lowfreq: posting ids
    uint64_t* results;                   // [n_routes][topk] idx_t
    float* distances;
    int* steps;
    uint32_t base_rows, dim, degree, n_routes, range_count, finish_count, max_steps, topk;
    int32_t early_stop_mode, queue_size, dtype, reserved;
};

namespace gofann_ref_full {

namespace fg = go_fann::backend_full_gpu;

template <int QS, typename T>
int launch_high(const gofann_ref_full_args& a)
{
    fg::full_gpu_highfreq_kernel<QS, T, false>
        <<<a.n_routes, fg::kHighfreqBlockThreads, static_cast<size_t>(a.dim) * sizeof(T)>>>(
            static_cast<const T*>(a.base), static_cast<const T*>(a.queries), a.base_rows, a.dim, a.graph, a.degree,
            a.degree, a.active_ids, a.n_routes, a.query_vector_ids, a.group_ids, a.start_local, a.label_size,
            a.label_offset, a.row_to_sample, a.row_filter_mask, a.filter_bits, a.filter_modes, a.single_extra,
            a.active_range_counts, a.qlabel_indptr, a.qlabel_indices, a.sample_indptr, a.sample_indices,
            a.range_modes, a.range_lower, a.range_upper, a.base_ranges, a.range_count, a.finish_count,
            a.early_stop_mode, a.max_steps, a.topk, reinterpret_cast<idx_t*>(a.results), a.distances, a.steps);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

template <typename T>
int by_queue(const gofann_ref_full_args& a)
{
    switch (a.queue_size) {
    case 16: return launch_high<16, T>(a);
    case 32: return launch_high<32, T>(a);
    case 48: return launch_high<48, T>(a);
    case 64: return launch_high<64, T>(a);
    case 96: return launch_high<96, T>(a);
    case 128: return launch_high<128, T>(a);
    case 192: return launch_high<192, T>(a);
    case 256: return launch_high<256, T>(a);
    case 384: return launch_high<384, T>(a);
    case 512: return launch_high<512, T>(a);
    default: return -1;
    }
}

template <typename T>
int launch_low(const gofann_ref_full_args& a)
{
    fg::full_gpu_lowfreq_kernel<T><<<a.n_routes, 32, static_cast<size_t>(a.dim) * sizeof(T)>>>(
        static_cast<const T*>(a.base), static_cast<const T*>(a.queries), a.base_rows, a.dim, a.active_ids,
        a.n_routes, a.query_vector_ids, a.group_ids, a.filter_bits, a.label_size, a.label_offset, a.low_sample_ids,
        a.row_filter_mask, a.filter_modes, a.single_extra, a.active_range_counts, a.qlabel_indptr, a.qlabel_indices,
        a.sample_indptr, a.sample_indices, a.range_modes, a.range_lower, a.range_upper, a.base_ranges,
        a.range_count, a.topk, reinterpret_cast<idx_t*>(a.results), a.distances, a.steps);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

__global__ void ref_block_pickup_cases(go_fann::warp_kernel::KernelPair<float, uint32_t>* frontiers,
                                       const int* sizes, int stride, int* picked)
{
    __shared__ int warp_best_indices[fg::kHighfreqBlockThreads / 32];
    __shared__ float warp_best_distances[fg::kHighfreqBlockThreads / 32];
    __shared__ int selected;
    auto* f = frontiers + static_cast<size_t>(blockIdx.x) * stride;
    go_fann::warp_kernel::KernelPair<float, uint32_t> out;
    const bool found = fg::pickup_next_unused_from_pool_block(f, sizes[blockIdx.x], out, warp_best_indices,
                                                          warp_best_distances, selected);
    if (threadIdx.x == 0) picked[blockIdx.x] = found ? static_cast<int>(out.second & 0x7fffffffu) : -1;
}

}  // namespace gofann_ref_full

using namespace gofann_ref_full;

extern "C" {

// Launches the reference's graph-route kernel on the legacy default stream;
// 0 = launched, -1 = a queue size the reference does not instantiate (it
// rounds other sizes up to one of these) or topk outside 1..10, -2 = launch
// error.
__attribute__((visibility("default"))) int gofann_ref_full_highfreq(const gofann_ref_full_args* a)
{
    if (!a || a->topk < 1 || a->topk > 10 || a->degree > 64) return -1;
    if (a->dtype == 0) return by_queue<uint8_t>(*a);
    if (a->dtype == 1) return by_queue<float>(*a);
    if (a->dtype == 2) return by_queue<__half>(*a);
    return -1;
}

__attribute__((visibility("default"))) int gofann_ref_full_lowfreq(const gofann_ref_full_args* a)
{
    if (!a || a->topk < 1 || a->topk > 10) return -1;
    if (a->dtype == 0) return launch_low<uint8_t>(*a);
    if (a->dtype == 1) return launch_low<float>(*a);
    if (a->dtype == 2) return launch_low<__half>(*a);
    return -1;
}

// The block pickup on crafted frontiers: frontier c has `stride` entries of
// (distance, payload = index | used << 31), heap size sizes[c]; picked[c]
// receives the payload index taken, or -1.
__attribute__((visibility("default"))) int gofann_ref_block_pickup_cases(void* frontiers, const int* sizes,
                                                                         int n_cases, int stride, int* picked)
{
    if (n_cases <= 0) return 0;
    ref_block_pickup_cases<<<n_cases, fg::kHighfreqBlockThreads>>>(
        static_cast<go_fann::warp_kernel::KernelPair<float, uint32_t>*>(frontiers), sizes, stride, picked);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

__attribute__((visibility("default"))) size_t gofann_ref_full_args_size(void) { return sizeof(gofann_ref_full_args); }

}  // extern "C"
