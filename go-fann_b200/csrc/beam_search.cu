// beam_search.cu — C-ABI entry points of the filtered graph beam search:
// argument checks, variant choice, launch sizing and the two traversal
// entry points (caller scratch, and the allocation-free one).  The kernel
// itself is in beam_kernel.cuh; its variants are instantiated in
// beam_variants_*.cu.
#include "beam_kernel.cuh"

#include <mutex>

namespace gofann {
namespace {

using beam::BeamArgs;
using beam::KernelFn;
using beam::SmemLayout;
using beam::kMaxBlockWarps;
using beam::kU8BlockWarps;
using beam::kWarpsPerBlock;

// ext: the routes' clauses carry string / integer atoms (a variant without
// their check otherwise)
KernelFn pick_kernel(int scorer, bool bias, int pq_mode, bool w4, bool small_m, bool ext)
{
    if (scorer != GOFANN_SCORER_PQ) return beam::pick_rabitq(bias, ext);
    switch (pq_mode) {
    case GOFANN_PQ_U8: return beam::pick_u8(bias, w4, small_m, ext);
    case GOFANN_PQ_DIRECT: return beam::pick_direct(bias, w4, small_m, ext);
    case GOFANN_PQ_LUT_SHARED: return beam::pick_table(true, bias, small_m, ext);
    default: return beam::pick_table(false, bias, small_m, ext);
    }
}

// Validates the PQ-mode specific inputs; sets w4 / small_m.
int check_pq_mode(const gofann_search_params& p, const gofann_codes& c, const gofann_prepared& prep, bool& w4,
                  bool& small_m, const char* who)
{
    w4 = false;
    small_m = c.pq_dim <= 64;
    if (p.pq_mode == GOFANN_PQ_DIRECT) {
        if (!prep.pq_query || !prep.pq_centroids || prep.dim == 0 || prep.dim % c.pq_dim != 0)
            return fail(GOFANN_ERR_INVALID, "%s: direct PQ scoring needs pq_query, pq_centroids and dim %% pq_dim == 0",
                        who);
        if (prep.pq_query_dtype != GOFANN_DTYPE_U8 && prep.pq_query_dtype != GOFANN_DTYPE_F32)
            return fail(GOFANN_ERR_INVALID, "%s: pq_query_dtype must be u8 or f32", who);
        if (prep.dim > 4096) return fail(GOFANN_ERR_UNSUPPORTED, "%s: dim %u above 4096", who, prep.dim);
        w4 = prep.dim / c.pq_dim == 4 && (reinterpret_cast<uintptr_t>(prep.pq_centroids) & 15) == 0;
        return GOFANN_OK;
    }
    if (p.pq_mode == GOFANN_PQ_U8) {
        if (!prep.pq_query || !prep.pq_centroids || prep.pq_query_dtype != GOFANN_DTYPE_U8 || prep.dim == 0 ||
            prep.dim % c.pq_dim != 0 || (prep.dim / c.pq_dim) % 4 != 0)
            return fail(GOFANN_ERR_INVALID,
                        "%s: u8 PQ scoring needs u8 pq_query, pq_centroids and dim / pq_dim a multiple of 4", who);
        if ((reinterpret_cast<uintptr_t>(prep.pq_query) & 3) != 0)
            return fail(GOFANN_ERR_INVALID, "%s: pq_query must be 4-byte aligned", who);
        if (prep.dim > 256) return fail(GOFANN_ERR_UNSUPPORTED, "%s: u8 PQ scoring needs dim <= 256", who);
        w4 = prep.dim / c.pq_dim == 4 && c.pq_dim % 16 == 0;  // the chunked scorer
        return GOFANN_OK;
    }
    if (p.pq_mode != GOFANN_PQ_LUT_GLOBAL && p.pq_mode != GOFANN_PQ_LUT_SHARED)
        return fail(GOFANN_ERR_INVALID, "%s: unknown pq_mode %d", who, p.pq_mode);
    if (!prep.pq_lut) return fail(GOFANN_ERR_INVALID, "%s: PQ lookup table missing", who);
    return GOFANN_OK;
}

// Persistent grid: at most one warp per route, at most what fits resident.
uint32_t grid_blocks(uint32_t n_routes, int warps_per_block, int per_sm)
{
    const uint32_t need = (n_routes + warps_per_block - 1) / warps_per_block;
    const uint32_t cap = static_cast<uint32_t>(per_sm > 0 ? per_sm : 1) * static_cast<uint32_t>(sm_count());
    return need < cap ? need : cap;
}

// Share of L2 that the automatic grid size lets the running routes' tables
// (lookup row + visited table per warp) occupy when the lookup tables are
// read from global memory; 0 disables the automatic cap.
constexpr double kAutoL2Share = 0.0;

// Routes in flight: an explicit resident_warps caps the grid; with 0, in
// GOFANN_PQ_LUT_GLOBAL mode the grid is cut to the warps whose tables fit in
// kAutoL2Share of L2 (never below one block per SM).
uint32_t cap_blocks(uint32_t blocks, const gofann_search_params& p, int wpb, int pq_mode, uint32_t pq_dim)
{
    uint64_t cap_warps = 0;
    if (p.resident_warps > 0) {
        cap_warps = static_cast<uint64_t>(p.resident_warps);
    } else if (p.scorer == GOFANN_SCORER_PQ && pq_mode == GOFANN_PQ_LUT_GLOBAL && kAutoL2Share > 0.0) {
        const uint64_t per_warp = static_cast<uint64_t>(pq_dim) * GOFANN_PQ_CENTROIDS * 4 + kHashCap * 4;
        cap_warps = static_cast<uint64_t>(kAutoL2Share * static_cast<double>(l2_bytes())) / per_warp;
        const uint64_t floor_warps = static_cast<uint64_t>(sm_count() > 0 ? sm_count() : 1) * wpb;
        if (cap_warps < floor_warps) cap_warps = floor_warps;
    }
    if (cap_warps == 0) return blocks;
    uint64_t cap = cap_warps / static_cast<uint64_t>(wpb);
    if (cap == 0) cap = 1;
    return blocks < cap ? blocks : static_cast<uint32_t>(cap);
}

constexpr size_t kCounterBytes = 256;  // route counter, kept 256-byte aligned

// A validated traversal call, sized for launch: the kernel arguments (the
// scratch pointers still unset), the variant, its block shape and shared
// memory, and the persistent grid before any scratch cap.
struct LaunchPlan {
    BeamArgs args;
    KernelFn kern;
    int wpb;
    size_t smem;
    uint32_t blocks;
};

// Checks a call's arguments (both traversal entry points share the rules and
// the messages, prefixed with `who`) and, when there are routes, picks the
// kernel variant and sizes its launch.
int plan_launch(const gofann_graph* graph, const gofann_attrs* attrs, const gofann_codes* codes,
                const gofann_prepared* prep, const gofann_routes* routes, const gofann_search_params* params,
                const gofann_search_out* out, const char* who, LaunchPlan& lp)
{
    if (!graph || !codes || !prep || !routes || !params || !out) return fail(GOFANN_ERR_INVALID, "%s: null argument", who);
    const gofann_search_params& p = *params;
    if (p.queue_size < 2 || p.queue_size > GOFANN_MAX_QUEUE)
        return fail(GOFANN_ERR_INVALID, "%s: queue_size %d outside 2..%d", who, p.queue_size, GOFANN_MAX_QUEUE);
    if (p.stop_width < 1 || p.stop_width > GOFANN_MAX_TOPK)
        return fail(GOFANN_ERR_INVALID, "%s: stop_width %d outside 1..%d", who, p.stop_width, GOFANN_MAX_TOPK);
    if (p.result_width < 1 || p.result_width > GOFANN_MAX_RESULT_WIDTH)
        return fail(GOFANN_ERR_INVALID, "%s: result_width %d outside 1..%d", who, p.result_width,
                    GOFANN_MAX_RESULT_WIDTH);
    if (p.early_stop_mode < 0 || p.early_stop_mode > 2)
        return fail(GOFANN_ERR_INVALID, "%s: unknown early_stop_mode %d", who, p.early_stop_mode);
    if (p.resident_warps < 0)
        return fail(GOFANN_ERR_INVALID, "%s: resident_warps %d is negative", who, p.resident_warps);
    if (!graph->adjacency || !graph->row_to_sample || !graph->label_offset || graph->degree == 0)
        return fail(GOFANN_ERR_INVALID, "%s: graph arrays missing", who);
    const uint32_t min_stride = GOFANN_RECORD_META(codes->pq_dim) + 16u + 4u * GOFANN_RECORD_INLINE_LABELS;
    if (graph->records && p.scorer == GOFANN_SCORER_PQ &&
        ((graph->record_stride & 15u) != 0 || (reinterpret_cast<uintptr_t>(graph->records) & 15) != 0 ||
         graph->record_stride < min_stride))
        return fail(GOFANN_ERR_INVALID, "%s: row records need 16-byte alignment and a stride of at least %u", who,
                    min_stride);
    if (!routes->query_row || !routes->group_id || !routes->start_local || !out->ids || !out->dists)
        return fail(GOFANN_ERR_INVALID, "%s: route or output arrays missing", who);
    const bool needs_attrs = routes->pred_offsets != nullptr || p.full_label_check != 0 ||
                             routes->range_modes != nullptr;
    if (needs_attrs && (!attrs || !attrs->label_indptr || !attrs->label_indices))
        return fail(GOFANN_ERR_INVALID, "%s: predicates need the sample label CSR", who);
    if (routes->pred_offsets && (!routes->clauses || !routes->pred_handles))
        return fail(GOFANN_ERR_INVALID, "%s: predicate clause arrays missing", who);
    int pq_mode = GOFANN_PQ_LUT_GLOBAL;
    bool w4 = false, small_m = true;
    if (p.scorer == GOFANN_SCORER_PQ) {
        if (!codes->pq_codes) return fail(GOFANN_ERR_INVALID, "%s: PQ codes missing", who);
        if (codes->pq_dim == 0 || codes->pq_dim > static_cast<uint32_t>(kMaxPqDim))
            return fail(GOFANN_ERR_UNSUPPORTED, "%s: pq_dim %u outside 1..%d", who, codes->pq_dim, kMaxPqDim);
        const int st = check_pq_mode(p, *codes, *prep, w4, small_m, who);
        if (st != GOFANN_OK) return st;
        pq_mode = p.pq_mode;
    } else if (p.scorer == GOFANN_SCORER_RABITQ) {
        if (!codes->rq_codes || !codes->rq_factors || !codes->rq_anchor_ids || !prep->rq_q8 || !prep->rq_scale ||
            !prep->rq_k1xsumq || !prep->rq_centroid_dist)
            return fail(GOFANN_ERR_INVALID, "%s: RaBitQ arrays missing", who);
        if (codes->padded_dim == 0 || codes->padded_dim % 64 != 0 || codes->padded_dim > 4096)
            return fail(GOFANN_ERR_UNSUPPORTED, "%s: padded_dim %u unsupported", who, codes->padded_dim);
    } else {
        return fail(GOFANN_ERR_INVALID, "%s: unknown scorer %d", who, p.scorer);
    }
    lp = LaunchPlan{};
    if (routes->n_routes == 0) return GOFANN_OK;

    BeamArgs& args = lp.args;
    args.graph = *graph;
    args.attrs = make_attr_view(attrs);
    args.codes = *codes;
    args.prep = *prep;
    args.routes = *routes;
    args.p = p;
    args.out = *out;
    args.status = out->status;
    const SmemLayout L = beam::smem_layout(p, *codes, pq_mode, prep->dim);
    args.warp_smem = L.total;
    // GOFANN_PQ_U8: the packed codebook ahead of the warps' areas
    const bool u8 = pq_mode == GOFANN_PQ_U8 && p.scorer == GOFANN_SCORER_PQ;
    args.block_smem = u8 ? static_cast<uint32_t>(codes->pq_dim * GOFANN_PQ_CENTROIDS * (prep->dim / codes->pq_dim))
                         : 0u;
    constexpr size_t kMaxSmem = 227 * 1024;
    int wpb = u8 ? kU8BlockWarps : kWarpsPerBlock;
    while (wpb > 1 && args.block_smem + static_cast<size_t>(L.total) * wpb > kMaxSmem) --wpb;
    const size_t smem = args.block_smem + static_cast<size_t>(L.total) * wpb;
    if (smem > kMaxSmem)
        return fail(GOFANN_ERR_UNSUPPORTED, "%s: %zu bytes of shared memory per warp exceed 227 KB", who, smem);
    const KernelFn kern = pick_kernel(p.scorer, p.predicate_bias != 0, pq_mode, w4, small_m,
                                      routes->pred_offsets != nullptr && routes->pred_ext != nullptr);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e, "beam_search: shared memory attribute");
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, wpb * 32, smem);
    if (e != cudaSuccess) return cuda_status(e, "beam_search: occupancy query");
    if (per_sm <= 0) return fail(GOFANN_ERR_UNSUPPORTED, "%s: kernel does not fit on an SM", who);
    lp.kern = kern;
    lp.wpb = wpb;
    lp.smem = smem;
    lp.blocks = cap_blocks(grid_blocks(routes->n_routes, wpb, per_sm), p, wpb, pq_mode, codes->pq_dim);
    return GOFANN_OK;
}

// Clears the route counter at the head of `scratch` and launches `blocks`
// persistent blocks whose warps take visited tables from after it.
int launch_planned(LaunchPlan& lp, uint32_t blocks, void* scratch, void* stream, const char* what)
{
    lp.args.route_counter = static_cast<uint32_t*>(scratch);
    lp.args.hash = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(scratch) + kCounterBytes);
    cudaStream_t s = as_stream(stream);
    cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(uint32_t), s);
    if (e != cudaSuccess) return cuda_status(e, "beam_search: counter reset");
    lp.kern<<<blocks, lp.wpb * 32, lp.smem, s>>>(lp.args);
    GOFANN_CHECK_LAUNCH(what);
    return GOFANN_OK;
}

}  // namespace
}  // namespace gofann

using namespace gofann;

extern "C" {

size_t gofann_beam_search_scratch_bytes(uint32_t n_routes)
{
    // Upper bound over variants: one table per warp of the persistent grid,
    // which never exceeds one warp per route nor 64 warps per SM.
    const uint32_t sms = static_cast<uint32_t>(sm_count() > 0 ? sm_count() : 148);
    // (the last block of a grid of ceil(n_routes / wpb) blocks adds < wpb warps)
    uint64_t warps = static_cast<uint64_t>(n_routes) + kMaxBlockWarps - 1;
    const uint64_t cap = static_cast<uint64_t>(sms) * 64;
    if (warps > cap) warps = cap;
    if (warps == 0) warps = kMaxBlockWarps;
    return kCounterBytes + warps * kHashCap * sizeof(uint32_t);
}

int gofann_beam_search(const gofann_graph* graph, const gofann_attrs* attrs, const gofann_codes* codes,
                       const gofann_prepared* prep, const gofann_routes* routes,
                       const gofann_search_params* params, const gofann_search_out* out, void* scratch,
                       size_t scratch_bytes, void* stream)
{
    if (!scratch) return fail(GOFANN_ERR_INVALID, "beam_search: null argument");
    LaunchPlan lp;
    const int st = plan_launch(graph, attrs, codes, prep, routes, params, out, "beam_search", lp);
    if (st != GOFANN_OK || routes->n_routes == 0) return st;
    const size_t need = kCounterBytes + static_cast<size_t>(lp.blocks) * lp.wpb * kHashCap * sizeof(uint32_t);
    if (scratch_bytes < need)
        return fail(GOFANN_ERR_CAPACITY, "beam_search: scratch of %zu bytes, %zu needed", scratch_bytes, need);
    return launch_planned(lp, lp.blocks, scratch, stream, "beam_search_kernel");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free traversal entry point.
//
// Some callers cannot allocate device memory at all: a host process whose
// device memory is owned by another allocator (a database or JVM/Go runtime
// embedding this library and handing it only pre-sized buffers), code that
// must not call cudaMalloc while another library is capturing its stream
// into a CUDA graph, or latency-critical serving paths where an allocation
// (and the device synchronisation cudaFree implies) is not acceptable.  For
// them the traversal's scratch -- the route counter and one 4096-slot
// visited table per resident warp -- lives in the file-scope device array
// below instead of a caller-supplied buffer.
//
// Limits and sharing: the array holds kNoAllocTables (1,024) visited tables,
// 16 MiB + 256 B, allocated once per device by the CUDA runtime when this
// library is loaded and held until the process exits.  At most 1,024 warps
// run at once in this mode (the grid is capped to that; any number of routes
// is still processed, since warps pull routes from the counter): with the
// 24-warp blocks of GOFANN_PQ_U8 that is 42 blocks, so 42 of a B200's 148
// SMs do the work and a large batch takes about 3.5x as long as through
// gofann_beam_search; the 4-warp blocks of the other modes fill 256 blocks.
// Every call on a device uses the same array, which keeps the previous
// call's contents: the counter is cleared before each launch and each warp
// clears its visited table per route, so nothing stale is read.  Calls
// whose kernels overlap on the GPU (different streams, or different host
// threads) race on the array and must be serialised by the caller.
//
// The array's device address is looked up once per device and cached for
// the life of the process; a device reset (cudaDeviceReset, or destroying
// the primary context) invalidates it and is not supported while this
// library is loaded.
namespace gofann {
namespace {
constexpr int kNoAllocTables = 1024;
constexpr size_t kNoAllocBytes = kCounterBytes + static_cast<size_t>(kNoAllocTables) * kHashCap * sizeof(uint32_t);
}  // namespace
}  // namespace gofann

static __device__ __align__(256) unsigned char g_noalloc_scratch[gofann::kNoAllocBytes];

namespace gofann {
namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_address[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  Host code may
// not pass the symbol itself to a kernel (in host code it names a host-side
// stand-in), so the address is looked up once per device, with that device
// current, on the first call.
int noalloc_scratch_address(void** out)
{
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "beam_search_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(GOFANN_ERR_UNSUPPORTED, "beam_search_noalloc: device %d outside 0..%d", dev, kNoAllocMaxDevices - 1);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_address[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_status(e, "beam_search_noalloc: cudaGetSymbolAddress");
        g_noalloc_address[dev] = p;
    }
    *out = g_noalloc_address[dev];
    return GOFANN_OK;
}

}  // namespace
}  // namespace gofann

extern "C" {

int gofann_beam_search_noalloc(const gofann_graph* graph, const gofann_attrs* attrs, const gofann_codes* codes,
                               const gofann_prepared* prep, const gofann_routes* routes,
                               const gofann_search_params* params, const gofann_search_out* out, void* stream)
{
    LaunchPlan lp;
    int st = plan_launch(graph, attrs, codes, prep, routes, params, out, "beam_search_noalloc", lp);
    if (st != GOFANN_OK) return st;
    void* scratch = nullptr;
    st = noalloc_scratch_address(&scratch);
    if (st != GOFANN_OK || routes->n_routes == 0) return st;
    const uint32_t max_blocks = static_cast<uint32_t>(kNoAllocTables / lp.wpb);
    const uint32_t blocks = lp.blocks < max_blocks ? lp.blocks : max_blocks;
    const size_t need = kCounterBytes + static_cast<size_t>(blocks) * lp.wpb * kHashCap * sizeof(uint32_t);
    if (blocks == 0 || need > kNoAllocBytes)
        return fail(GOFANN_ERR_CAPACITY,
                    "beam_search_noalloc: %zu bytes of scratch needed, the static scratch holds %zu (%d visited tables)",
                    need, kNoAllocBytes, kNoAllocTables);
    return launch_planned(lp, blocks, scratch, stream, "beam_search_kernel (no-alloc)");
}

}  // extern "C"
