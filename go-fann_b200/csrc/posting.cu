// posting.cu — brute-force scans of label postings and attribute-order
// slices, fused DNF filter, top-shortlist by (dist, id).
//
// The reference scans one route per single-thread block, inserting into a
// (dist, id) max-heap one candidate at a time (lowfreq_pq_scan_kernel,
// src/search/pq/backend_pq.cu:2046-2185; RaBitQ twin backend_rabitq.cu:
// 5396-5751).  That heap ends holding exactly the k smallest (dist, id)
// pairs of the passing candidates, whatever the insertion order, and its
// score-first elision only skips candidates that cannot enter.  Here one
// 256-thread block scores a route's candidates in parallel and keeps the k
// smallest pairs with a threshold filter: a candidate enters a shared-memory
// buffer only when it is below the k-th pair of the candidates merged so far
// (so it could still be in the result), and a full buffer is merged into the
// running top-k by a bitonic sort.  After the first merge only about
// k ln(n / k) of n candidates pass, so sorting costs little next to scoring.
//
// Scorers:
//  * PQ tables: the query's LUT row (given, or built per route from the
//    codebook as computePQTable does inside the reference's scan) staged in
//    shared memory; the sum is sequential over subspaces
//    (backend_pq.cu:2101-2104), one candidate per thread;
//  * PQ_U8 (u8 queries, integer codebook): every table entry and partial sum
//    is an integer below 2^24, so the sequential float sum equals the
//    integer sum of byte differences against a packed codebook.  The blocks
//    are persistent: each packs the codebook into shared memory once and
//    then scans routes blockIdx.x, blockIdx.x + gridDim.x, ... -- no
//    per-route table or codebook read;
//  * RaBitQ: padded_dim = 128 G (G = 1..32) gives each candidate G lanes;
//    a lane reads 16 bytes of the code (one coalesced 16 G-byte row per
//    candidate) against its 4 words of the query's bit planes, held in
//    registers for the whole route, and the lanes' partial inner products
//    are summed by a warp reduction.  Other padded dims score one candidate
//    per thread against the planes in shared memory.
#include "exact_device.cuh"
#include "pq_device.cuh"
#include "rq_device.cuh"

namespace gofann {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanWarps = kScanThreads / kWarp;
constexpr int kSortSize = 2048;      // running top-k + buffer, sorted together
constexpr int kBatches = 4;          // 32-candidate batches per warp between buffer checks
constexpr int kRoundCands = kScanWarps * kWarp * kBatches;

// kScanExact*: exact L2 of the full base rows (the Full-GPU backend's
// low-frequency scan, full_gpu_lowfreq_kernel, backend_full_gpu.cu:
// 2124-2260), one candidate per thread.
enum ScanKind { kScanPqTable = 0, kScanPqU8 = 1, kScanRabitq = 2, kScanExactU8 = 3, kScanExactF32 = 4,
                kScanExactF16 = 5 };
template <int kKind>
constexpr bool is_exact() { return kKind == kScanExactU8 || kKind == kScanExactF32 || kKind == kScanExactF16; }

__device__ __forceinline__ void bitonic_sort_pairs(float* d, uint32_t* id, int n, int tid)
{
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < n / 2; i += kScanThreads) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = (lo & size) == 0;
                const float dl = d[lo], dh = d[hi];
                const uint32_t il = id[lo], ih = id[hi];
                const bool greater = pair_less(dh, ih, dl, il);  // lo > hi
                if (greater == up) { d[lo] = dh; d[hi] = dl; id[lo] = ih; id[hi] = il; }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ uint32_t next_pow2(uint32_t x)
{
    return x <= 1 ? 1u : 1u << (32 - __clz(x - 1));
}

// Running top-k of one route: sorted pairs at [0, keep), the buffer after
// them.  Empty slots hold (FLT_MAX, UINT32_MAX), the fill of the
// reference's shortlist heap, which is also the first threshold: a
// candidate enters only below it, as it enters that heap.
struct TopK {
    float* sd;
    uint32_t* sid;
    int keep, k;
};
struct TopKState {
    int n_buf;
    float thr_d;
    uint32_t thr_id;
    int fresh;  // 1 until the first merge: the top-k holds only the fill
};

__device__ __forceinline__ void topk_reset(const TopK& t, TopKState& st, int tid)
{
    for (int i = tid; i < t.keep; i += kScanThreads) { t.sd[i] = FLT_MAX; t.sid[i] = kU32Max; }
    if (tid == 0) { st.n_buf = 0; st.thr_d = FLT_MAX; st.thr_id = kU32Max; st.fresh = 1; }
    __syncthreads();
}

// Buffers (d, s) when it is below the threshold pair (the k-th smallest pair
// merged so far, or the sentinel before k candidates were merged).
__device__ __forceinline__ void topk_offer(const TopK& t, TopKState& st, float thr_d, uint32_t thr_id, float d,
                                           uint32_t s)
{
    if (pair_less(d, s, thr_d, thr_id)) {
        const int p = atomicAdd(&st.n_buf, 1);
        t.sd[t.keep + p] = d;
        t.sid[t.keep + p] = s;
    }
}

// Sorts the top-k and `n_buf` buffered pairs (block-uniform n_buf).  At
// the first merge the top-k holds only the fill, so only the buffer is
// sorted (in place, padded with the fill to a power of two) and its first
// `keep` pairs become the top-k: a short route sorts its own candidates
// instead of keep + n_buf pairs.
__device__ __forceinline__ void topk_merge(const TopK& t, TopKState& st, int n_buf, int tid)
{
    const int fresh = st.fresh;
    const int nb2 = static_cast<int>(next_pow2(static_cast<uint32_t>(n_buf)));
    if (fresh && t.keep + nb2 <= kSortSize) {
        float* bd = t.sd + t.keep;
        uint32_t* bi = t.sid + t.keep;
        for (int i = n_buf + tid; i < nb2; i += kScanThreads) { bd[i] = FLT_MAX; bi[i] = kU32Max; }
        __syncthreads();
        bitonic_sort_pairs(bd, bi, nb2, tid);
        for (int i = tid; i < t.keep; i += kScanThreads) {
            t.sd[i] = i < nb2 ? bd[i] : FLT_MAX;
            t.sid[i] = i < nb2 ? bi[i] : kU32Max;
        }
        __syncthreads();
        if (tid == 0) { st.n_buf = 0; st.thr_d = t.sd[t.k - 1]; st.thr_id = t.sid[t.k - 1]; st.fresh = 0; }
        __syncthreads();
        return;
    }
    const int n = t.keep + n_buf;
    const int np2 = static_cast<int>(next_pow2(static_cast<uint32_t>(n)));
    for (int i = n + tid; i < np2; i += kScanThreads) { t.sd[i] = FLT_MAX; t.sid[i] = kU32Max; }
    __syncthreads();
    bitonic_sort_pairs(t.sd, t.sid, np2, tid);
    if (tid == 0) { st.n_buf = 0; st.thr_d = t.sd[t.k - 1]; st.thr_id = t.sid[t.k - 1]; st.fresh = 0; }
    __syncthreads();
}

// Posting id at position i of the route, or UINT32_MAX when it fails the
// route's predicate.
__device__ __forceinline__ uint32_t scan_candidate(const gofann_routes& routes, const AttrView& attrs,
                                                   uint32_t route, bool pred_on,
                                                   const uint32_t* __restrict__ posting_ids, uint64_t begin,
                                                   uint32_t i, uint32_t count)
{
    uint32_t s = kU32Max;
    if (i < count) {
        s = __ldg(posting_ids + begin + i);
        if (s != kU32Max && pred_on && !pred_matches(routes, attrs, route, s)) s = kU32Max;
    }
    return s;
}

// 16-byte streaming load (read once per route: L2 evict-first).
__device__ __forceinline__ uint4 ld_stream_u32x4(const void* p, uint64_t pol)
{
    return ldg_u32x4(reinterpret_cast<const uint4*>(p), pol);
}

template <int kG>
__device__ __forceinline__ int32_t group_sum(int32_t v)
{
    if constexpr (kG == 32) {
        return __reduce_add_sync(kFull, v);
    } else {
#pragma unroll
        for (int o = kG / 2; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
        return v;
    }
}

struct ScanArgs;
template <int kKind>
__device__ __forceinline__ void prefetch_candidate(const ScanArgs& a, uint32_t s);

struct ScanArgs {
    gofann_codes codes;
    gofann_prepared prep;
    AttrView attrs;
    gofann_routes routes;
    const uint32_t* posting_ids;
    const uint64_t* route_begin;
    const uint32_t* route_count;
    int k;
    uint32_t* out_ids;
    float* out_d;
    int32_t* status;
    const void* base;       // exact kinds: [n_samples][dim] rows
    const void* queries;    // exact kinds: [rows][dim]
    uint32_t dim;
    uint32_t row_bytes;
};

// Fetches candidate s's code row (and RaBitQ factors and anchor id) into
// L2 ahead of its scoring.
template <int kKind>
__device__ __forceinline__ void prefetch_candidate(const ScanArgs& a, uint32_t s)
{
    if (s == kU32Max) return;
    if constexpr (is_exact<kKind>()) {
        const unsigned char* p = static_cast<const unsigned char*>(a.base) + static_cast<size_t>(s) * a.row_bytes;
        for (uint32_t o = 0; o < a.row_bytes; o += 128) prefetch_l2(p + o);
    } else if constexpr (kKind == kScanRabitq) {
        const size_t cb = a.codes.padded_dim / 8;
        const uint8_t* p = a.codes.rq_codes + static_cast<size_t>(s) * cb;
        for (size_t o = 0; o < cb; o += 128) prefetch_l2(p + o);
        prefetch_l2(a.codes.rq_factors + static_cast<size_t>(s) * 3);
        prefetch_l2(a.codes.rq_anchor_ids + s);
    } else {
        const uint8_t* p = a.codes.pq_codes + static_cast<size_t>(s) * a.codes.pq_dim;
        prefetch_l2(p);
        prefetch_l2(p + a.codes.pq_dim - 1);
    }
}

// Three blocks per SM for the register-plane RaBitQ scorer (its 32 plane
// registers would otherwise leave two).
template <int kKind, int kG>
constexpr int scan_min_blocks() { return kKind == kScanRabitq && kG > 0 ? 3 : 1; }

// kKind: ScanKind; kG: lanes per RaBitQ candidate (0 = one thread each).
template <int kKind, int kG>
__global__ void __launch_bounds__(kScanThreads, scan_min_blocks<kKind, kG>()) posting_scan_kernel(ScanArgs a)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ TopKState st;
    __shared__ int s_bad;
    float* sd = reinterpret_cast<float*>(smem_raw);
    uint32_t* sid = reinterpret_cast<uint32_t*>(smem_raw + kSortSize * sizeof(float));
    uint32_t* wlist = sid + kSortSize;                                   // [kScanWarps][32]
    int32_t* wipbuf = reinterpret_cast<int32_t*>(wlist + kScanWarps * kWarp);  // [kScanWarps][32]
    unsigned char* area = reinterpret_cast<unsigned char*>(wipbuf + kScanWarps * kWarp);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int pq_dim = static_cast<int>(a.codes.pq_dim);
    const uint64_t stream_pol = l2_stream_policy();
    int keep = 32;
    while (keep < a.k) keep <<= 1;
    const TopK t{sd, sid, keep, a.k};
    const int cap = kSortSize - keep;

    // PQ_U8: pack the integer codebook once per (persistent) block
    uint32_t* cbw = reinterpret_cast<uint32_t*>(area);
    uint32_t* qw = cbw + pq_dim * GOFANN_PQ_CENTROIDS * (kKind == kScanPqU8 ? static_cast<int>(a.prep.dim) / pq_dim / 4
                                                                             : 0);
    if constexpr (kKind == kScanPqU8) {
        if (tid == 0) s_bad = 0;
        __syncthreads();
        const bool ok = pack_u8_codebook(a.prep.pq_centroids, static_cast<int>(a.prep.dim), pq_dim, cbw, tid,
                                         kScanThreads);
        if (!ok) s_bad = 1;
        __syncthreads();
        if (s_bad && tid == 0 && a.status) atomicExch(a.status, GOFANN_ERR_INVALID);
    }

    for (uint32_t route = blockIdx.x; route < a.routes.n_routes; route += gridDim.x) {
        const uint32_t row = a.routes.query_row[route];
        const bool pred_on = pred_enabled(a.routes, route);
        const uint64_t begin = a.route_begin[route];
        uint32_t count = a.route_count[route];
        if constexpr (kKind == kScanPqU8) {
            if (s_bad) count = 0;  // invalid codebook: empty results, status set
        }
        // ---- per-route query state
        float* table = reinterpret_cast<float*>(area);
        RqQueryView rq{};
        if constexpr (kKind == kScanPqTable) {
            const int dim = static_cast<int>(a.prep.dim);
            if (a.prep.pq_lut) {
                const float4* g = reinterpret_cast<const float4*>(a.prep.pq_lut + static_cast<size_t>(row) * pq_dim *
                                                                                      GOFANN_PQ_CENTROIDS);
                float4* t4 = reinterpret_cast<float4*>(table);
                for (int i = tid; i < pq_dim * GOFANN_PQ_CENTROIDS / 4; i += kScanThreads) t4[i] = __ldg(g + i);
            } else {
                // fused table build (computePQTable, backend_pq.cu:1999-2022, which
                // the reference also runs inside its scan): query row to shared
                // memory, then thread c evaluates column c of every subspace
                float* q = table + pq_dim * GOFANN_PQ_CENTROIDS;
                if (a.prep.pq_query_dtype == GOFANN_DTYPE_U8) {
                    const uint8_t* qr = static_cast<const uint8_t*>(a.prep.pq_query) + static_cast<size_t>(row) * dim;
                    for (int i = tid; i < dim; i += kScanThreads) q[i] = static_cast<float>(qr[i]);
                } else {
                    const float* qr = static_cast<const float*>(a.prep.pq_query) + static_cast<size_t>(row) * dim;
                    for (int i = tid; i < dim; i += kScanThreads) q[i] = qr[i];
                }
                __syncthreads();
                const int w = dim / pq_dim;
                const float* crow = a.prep.pq_centroids + static_cast<size_t>(tid) * dim;  // kScanThreads == 256
                const uint64_t keep_pol = l2_keep_policy();  // the codebook is shared by every route
                for (int m = 0; m < pq_dim; ++m)
                    table[m * GOFANN_PQ_CENTROIDS + tid] = pq_entry<0>(q + m * w, crow + m * w, w, keep_pol);
            }
        } else if constexpr (kKind == kScanPqU8) {
            const int nw = static_cast<int>(a.prep.dim) / 4;
            const uint32_t* qr = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(a.prep.pq_query) +
                                                                   static_cast<size_t>(row) * a.prep.dim);
            for (int i = tid; i < nw; i += kScanThreads) qw[i] = __ldg(qr + i);
        } else if constexpr (is_exact<kKind>()) {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(a.queries) +
                                                              static_cast<size_t>(row) * a.row_bytes);
            for (uint32_t i = tid; i < a.row_bytes / 16; i += kScanThreads)
                reinterpret_cast<uint4*>(area)[i] = __ldg(src + i);
        } else {
            rq_build_planes(a.prep.rq_q8 + static_cast<size_t>(row) * a.codes.padded_dim,
                            static_cast<int>(a.codes.padded_dim), reinterpret_cast<uint32_t*>(area), tid,
                            kScanThreads);
            rq.planes = reinterpret_cast<const uint32_t*>(area);
            rq.scale = a.prep.rq_scale[row];
            rq.k1 = a.prep.rq_k1xsumq[row];
            rq.gdist = a.prep.rq_centroid_dist + static_cast<size_t>(row) * a.codes.num_anchors;
        }
        topk_reset(t, st, tid);  // ends with a barrier: the query state is visible

        // RaBitQ group path: this lane's 4 plane words of every plane
        [[maybe_unused]] uint32_t pl[8][4];
        [[maybe_unused]] const int slot = kG > 0 ? lane % (kG > 0 ? kG : 1) : 0;
        if constexpr (kKind == kScanRabitq && kG > 0) {
            const int words = static_cast<int>(a.codes.padded_dim / 32);
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const uint4 v = *reinterpret_cast<const uint4*>(rq.planes + b * words + 4 * slot);
                pl[b][0] = v.x; pl[b][1] = v.y; pl[b][2] = v.z; pl[b][3] = v.w;
            }
        }

        // A warp scans positions warp*32 + 256 j (j = 0, 1, ...).  Without a
        // predicate, the ids of its next batch are loaded while this batch is
        // scored and their rows prefetched after it, one batch ahead.
        uint32_t s_next = kU32Max;
        bool have_next = false;
        for (uint32_t r0 = 0; r0 < count; r0 += kRoundCands) {
            const float thr_d = st.thr_d;
            const uint32_t thr_id = st.thr_id;
#pragma unroll 1
            for (int bt = 0; bt < kBatches; ++bt) {
                const uint32_t pos0 = r0 + static_cast<uint32_t>((bt * kScanWarps + warp) * kWarp);
                if (pos0 >= count) break;  // warp-uniform
                uint32_t s;
                if (have_next) {
                    s = s_next;
                } else {
                    s = scan_candidate(a.routes, a.attrs, route, pred_on, a.posting_ids, begin, pos0 + lane, count);
                    prefetch_candidate<kKind>(a, s);
                }
                have_next = !pred_on;
                if (have_next) {
                    const uint32_t pn = pos0 + kScanWarps * kWarp + lane;
                    s_next = pn < count ? __ldg(a.posting_ids + begin + pn) : kU32Max;
                }
                if constexpr (kKind == kScanRabitq && kG > 0) {
                    // Each lane loads the factors and anchor of its own candidate;
                    // the groups compute the inner products of the batch's live
                    // candidates in order (lane 0 of a group stores them); then
                    // every lane combines its own candidate's distance.
                    constexpr int kCpw = 32 / kG;                    // candidates per warp pass
                    constexpr int kU = kG >= 4 ? 4 : kG;             // passes unrolled
                    const unsigned live = __ballot_sync(kFull, s != kU32Max);
                    uint32_t* wl = wlist + warp * kWarp;
                    int32_t* wip = wipbuf + warp * kWarp;
                    const int my_pos = __popc(live & ((1u << lane) - 1u));
                    float fa = 0.0f, fr = 0.0f;
                    uint32_t an = 0u;
                    if (s != kU32Max) {
                        wl[my_pos] = s;
                        fa = __ldg(a.codes.rq_factors + static_cast<size_t>(s) * 3);
                        fr = __ldg(a.codes.rq_factors + static_cast<size_t>(s) * 3 + 1);
                        an = __ldg(a.codes.rq_anchor_ids + s);
                    }
                    __syncwarp();
                    const int n_live = __popc(live);
                    const int g = lane / kG;
                    const size_t code_bytes = a.codes.padded_dim / 8;
                    for (int j0 = 0; j0 < n_live; j0 += kCpw * kU) {
                        uint4 x[kU];
#pragma unroll
                        for (int u = 0; u < kU; ++u) {
                            const int j = j0 + u * kCpw + g;
                            x[u] = make_uint4(0u, 0u, 0u, 0u);
                            if (j < n_live)
                                x[u] = ld_stream_u32x4(a.codes.rq_codes + static_cast<size_t>(wl[j]) * code_bytes +
                                                           16 * slot,
                                                       stream_pol);
                        }
#pragma unroll
                        for (int u = 0; u < kU; ++u) {
                            const uint32_t cw[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
                            const int32_t ip = group_sum<kG>(rq_ip4_csa(cw, pl));
                            const int j = j0 + u * kCpw + g;
                            if (slot == 0 && j < n_live) wip[j] = ip;
                        }
                    }
                    __syncwarp();
                    if (s != kU32Max) {
                        const float d = rq_combine(wip[my_pos], rq.scale, rq.k1, fa, fr, __ldg(rq.gdist + an));
                        topk_offer(t, st, thr_d, thr_id, d, s);
                    }
                    __syncwarp();  // wl is rewritten by the next batch
                } else {
                    if (s != kU32Max) {
                        float d;
                        if constexpr (kKind == kScanPqTable) {
                            d = pq_adc_sequential(table, a.codes.pq_codes + static_cast<size_t>(s) * pq_dim, pq_dim);
                        } else if constexpr (kKind == kScanPqU8) {
                            d = pq_adc_u8_chunked(qw, cbw, a.codes.pq_codes + static_cast<size_t>(s) * pq_dim, pq_dim,
                                                  stream_pol);
                        } else if constexpr (kKind == kScanExactU8) {
                            d = static_cast<float>(l2_u8_thread(
                                static_cast<const uint8_t*>(a.base) + static_cast<size_t>(s) * a.row_bytes,
                                reinterpret_cast<const uint4*>(area), static_cast<int>(a.row_bytes / 16), stream_pol));
                        } else if constexpr (kKind == kScanExactF32 || kKind == kScanExactF16) {
                            d = l2_float_thread<kKind == kScanExactF32 ? GOFANN_DTYPE_F32 : GOFANN_DTYPE_F16>(
                                static_cast<const unsigned char*>(a.base) + static_cast<size_t>(s) * a.row_bytes, area,
                                static_cast<int>(a.dim));
                        } else {
                            d = rq_estimate(a.codes, rq, s);
                        }
                        topk_offer(t, st, thr_d, thr_id, d, s);
                    }
                }
                if (have_next) prefetch_candidate<kKind>(a, s_next);
            }
            __syncthreads();
            const int n_buf = st.n_buf;
            __syncthreads();  // every thread has read n_buf before a merge resets it
            if (n_buf > cap - kRoundCands) topk_merge(t, st, n_buf, tid);
        }
        {
            const int n_buf = st.n_buf;  // stable: the last round ended with barriers
            if (n_buf > 0) topk_merge(t, st, n_buf, tid);
        }
        for (int i = tid; i < a.k; i += kScanThreads) {
            const uint32_t id = sid[i];
            a.out_ids[static_cast<size_t>(route) * a.k + i] = id;
            a.out_d[static_cast<size_t>(route) * a.k + i] = id == kU32Max ? FLT_MAX : sd[i];
        }
        __syncthreads();  // the next route overwrites the shared state
    }
}

// Merge of segment shortlists (merge_shortlists, src/search/common/
// posting_segment_merge.cuh:13-61): route r's segments are rows
// seg_indptr[r] .. seg_indptr[r+1] of the [segments][k] shortlists; the
// reference inserts every entry into one k-slot shortlist heap, which keeps
// the k smallest (dist, id) pairs of the union -- what the threshold filter
// and the bitonic merges of TopK keep.
__global__ void __launch_bounds__(kScanThreads) segment_merge_kernel(const uint32_t* __restrict__ seg_indptr,
                                                                     uint32_t n_routes,
                                                                     const uint32_t* __restrict__ seg_ids,
                                                                     const float* __restrict__ seg_d, int k,
                                                                     uint32_t* __restrict__ out_ids,
                                                                     float* __restrict__ out_d)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ TopKState st;
    float* sd = reinterpret_cast<float*>(smem_raw);
    uint32_t* sid = reinterpret_cast<uint32_t*>(smem_raw + kSortSize * sizeof(float));
    const int tid = threadIdx.x;
    int keep = 32;
    while (keep < k) keep <<= 1;
    const TopK t{sd, sid, keep, k};
    const int cap = kSortSize - keep;
    for (uint32_t route = blockIdx.x; route < n_routes; route += gridDim.x) {
        const uint64_t b = static_cast<uint64_t>(seg_indptr[route]) * k;
        const uint64_t e = static_cast<uint64_t>(seg_indptr[route + 1]) * k;
        topk_reset(t, st, tid);
        for (uint64_t r0 = b; r0 < e; r0 += kRoundCands) {
            const float thr_d = st.thr_d;
            const uint32_t thr_id = st.thr_id;
            for (int j = tid; j < kRoundCands; j += kScanThreads) {
                const uint64_t i = r0 + j;
                if (i < e) topk_offer(t, st, thr_d, thr_id, __ldg(seg_d + i), __ldg(seg_ids + i));
            }
            __syncthreads();
            const int n_buf = st.n_buf;
            __syncthreads();
            if (n_buf > cap - kRoundCands) topk_merge(t, st, n_buf, tid);
        }
        {
            const int n_buf = st.n_buf;
            if (n_buf > 0) topk_merge(t, st, n_buf, tid);
        }
        for (int i = tid; i < k; i += kScanThreads) {
            const uint32_t id = sid[i];
            out_ids[static_cast<size_t>(route) * k + i] = id;
            out_d[static_cast<size_t>(route) * k + i] = id == kU32Max ? FLT_MAX : sd[i];
        }
        __syncthreads();
    }
}

template <int kKind, int kG>
int launch_scan(const ScanArgs& a, size_t smem, bool persistent, cudaStream_t s, const char* what)
{
    const auto kern = posting_scan_kernel<kKind, kG>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e, "posting_scan: shared memory attribute");
    unsigned blocks = a.routes.n_routes;
    if (persistent) {
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kScanThreads, smem);
        if (e != cudaSuccess) return cuda_status(e, "posting_scan: occupancy");
        const int sms = sm_count() > 0 ? sm_count() : 148;
        const unsigned full = static_cast<unsigned>((per_sm > 0 ? per_sm : 1) * sms);
        if (full < blocks) blocks = full;
    }
    kern<<<blocks, kScanThreads, smem, s>>>(a);
    GOFANN_CHECK_LAUNCH(what);
    return GOFANN_OK;
}

}  // namespace
}  // namespace gofann

using namespace gofann;

extern "C" {

int gofann_posting_scan(const gofann_codes* codes, const gofann_prepared* prep, const gofann_attrs* attrs,
                        const gofann_routes* routes, int scorer, const uint32_t* posting_ids,
                        const uint64_t* route_begin, const uint32_t* route_count, int32_t shortlist_k,
                        int32_t score_first, int32_t pq_mode, uint32_t* out_ids, float* out_dists,
                        int32_t* status, void* stream)
{
    (void)score_first;  // identical results either way (see file comment)
    if (!codes || !prep || !routes || !posting_ids || !route_begin || !route_count || !out_ids || !out_dists)
        return fail(GOFANN_ERR_INVALID, "posting_scan: null argument");
    if (shortlist_k < 1 || shortlist_k > GOFANN_MAX_SHORTLIST)
        return fail(GOFANN_ERR_INVALID, "posting_scan: shortlist %d outside 1..%d", shortlist_k, GOFANN_MAX_SHORTLIST);
    if (!routes->query_row) return fail(GOFANN_ERR_INVALID, "posting_scan: routes.query_row missing");
    if (routes->pred_offsets && (!attrs || !attrs->label_indptr || !routes->clauses || !routes->pred_handles))
        return fail(GOFANN_ERR_INVALID, "posting_scan: predicate arrays missing");
    if (routes->n_routes == 0) return GOFANN_OK;
    ScanArgs a{};
    a.codes = *codes;
    a.prep = *prep;
    a.routes = *routes;
    a.attrs = make_attr_view(attrs);
    a.posting_ids = posting_ids;
    a.route_begin = route_begin;
    a.route_count = route_count;
    a.k = shortlist_k;
    a.out_ids = out_ids;
    a.out_d = out_dists;
    a.status = status;
    const size_t base = static_cast<size_t>(kSortSize) * 8 + static_cast<size_t>(kScanWarps) * kWarp * 8;
    cudaStream_t s = as_stream(stream);
    if (scorer == GOFANN_SCORER_PQ) {
        if (!codes->pq_codes) return fail(GOFANN_ERR_INVALID, "posting_scan: PQ codes missing");
        if (codes->pq_dim == 0 || codes->pq_dim > static_cast<uint32_t>(kMaxPqDim))
            return fail(GOFANN_ERR_UNSUPPORTED, "posting_scan: pq_dim %u unsupported", codes->pq_dim);
        if (pq_mode == GOFANN_PQ_U8) {
            if (!prep->pq_query || !prep->pq_centroids || prep->pq_query_dtype != GOFANN_DTYPE_U8)
                return fail(GOFANN_ERR_INVALID, "posting_scan: PQ_U8 needs u8 pq_query and pq_centroids");
            if (prep->dim != 4 * codes->pq_dim || codes->pq_dim % 16 != 0 || prep->dim > 256)
                return fail(GOFANN_ERR_UNSUPPORTED,
                            "posting_scan: PQ_U8 needs 4-wide subvectors, pq_dim a multiple of 16 and dim <= 256 "
                            "(dim %u, pq_dim %u)", prep->dim, codes->pq_dim);
            if ((reinterpret_cast<uintptr_t>(codes->pq_codes) & 15) != 0 ||
                (reinterpret_cast<uintptr_t>(prep->pq_query) & 3) != 0)
                return fail(GOFANN_ERR_INVALID, "posting_scan: PQ_U8 needs 16-byte aligned codes, 4-byte aligned "
                                                "queries");
            const size_t smem = base + static_cast<size_t>(codes->pq_dim) * GOFANN_PQ_CENTROIDS * 4 + prep->dim;
            return launch_scan<kScanPqU8, 0>(a, smem, true, s, "posting_scan_kernel(u8)");
        }
        size_t table_bytes = static_cast<size_t>(codes->pq_dim) * GOFANN_PQ_CENTROIDS * sizeof(float);
        if (!prep->pq_lut) {
            if (!prep->pq_query || !prep->pq_centroids || prep->dim == 0 || prep->dim % codes->pq_dim != 0 ||
                prep->dim > 4096)
                return fail(GOFANN_ERR_INVALID, "posting_scan: needs pq_lut, or pq_query + pq_centroids + dim");
            table_bytes += static_cast<size_t>(prep->dim) * sizeof(float);
        }
        return launch_scan<kScanPqTable, 0>(a, base + table_bytes, false, s, "posting_scan_kernel(pq)");
    }
    if (scorer == GOFANN_SCORER_RABITQ) {
        if (!codes->rq_codes || !prep->rq_q8) return fail(GOFANN_ERR_INVALID, "posting_scan: RaBitQ arrays missing");
        const uint32_t pd = codes->padded_dim;
        if (pd == 0 || pd % 64 != 0 || pd > 4096)
            return fail(GOFANN_ERR_UNSUPPORTED, "posting_scan: padded_dim %u unsupported", pd);
        const size_t smem = base + pd;  // 8 planes of pd bits
        const bool aligned = (reinterpret_cast<uintptr_t>(codes->rq_codes) & 15) == 0;
        if (aligned && pd % 128 == 0) {
            switch (pd / 128) {
            case 1: return launch_scan<kScanRabitq, 1>(a, smem, false, s, "posting_scan_kernel(rq1)");
            case 2: return launch_scan<kScanRabitq, 2>(a, smem, false, s, "posting_scan_kernel(rq2)");
            case 4: return launch_scan<kScanRabitq, 4>(a, smem, false, s, "posting_scan_kernel(rq4)");
            case 8: return launch_scan<kScanRabitq, 8>(a, smem, false, s, "posting_scan_kernel(rq8)");
            case 16: return launch_scan<kScanRabitq, 16>(a, smem, false, s, "posting_scan_kernel(rq16)");
            case 32: return launch_scan<kScanRabitq, 32>(a, smem, false, s, "posting_scan_kernel(rq32)");
            default: break;
            }
        }
        return launch_scan<kScanRabitq, 0>(a, smem, false, s, "posting_scan_kernel(rq)");
    }
    return fail(GOFANN_ERR_INVALID, "posting_scan: unknown scorer %d", scorer);
}

int gofann_exact_posting_scan(const void* base, int dtype, uint32_t n_samples, uint32_t dim, const void* queries,
                              const gofann_attrs* attrs, const gofann_routes* routes, const uint32_t* posting_ids,
                              const uint64_t* route_begin, const uint32_t* route_count, int32_t k,
                              uint32_t* out_ids, float* out_dists, void* stream)
{
    if (!base || !queries || !routes || !posting_ids || !route_begin || !route_count || !out_ids || !out_dists)
        return fail(GOFANN_ERR_INVALID, "exact_posting_scan: null argument");
    if (k < 1 || k > GOFANN_MAX_SHORTLIST)
        return fail(GOFANN_ERR_INVALID, "exact_posting_scan: k %d outside 1..%d", k, GOFANN_MAX_SHORTLIST);
    if (!routes->query_row) return fail(GOFANN_ERR_INVALID, "exact_posting_scan: routes.query_row missing");
    if (routes->pred_offsets && (!attrs || !attrs->label_indptr || !routes->clauses || !routes->pred_handles))
        return fail(GOFANN_ERR_INVALID, "exact_posting_scan: predicate arrays missing");
    if (dtype != GOFANN_DTYPE_U8 && dtype != GOFANN_DTYPE_F32 && dtype != GOFANN_DTYPE_F16)
        return fail(GOFANN_ERR_INVALID, "exact_posting_scan: unknown dtype %d", dtype);
    const uint32_t elem = dtype == GOFANN_DTYPE_U8 ? 1u : (dtype == GOFANN_DTYPE_F16 ? 2u : 4u);
    if (dim == 0 || (dim * elem) % 16 != 0 || dim * elem > 16384)
        return fail(GOFANN_ERR_UNSUPPORTED, "exact_posting_scan: rows of %u x %u bytes (need a multiple of 16, "
                                            "<= 16 KB)", dim, elem);
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (reinterpret_cast<uintptr_t>(queries) & 15) != 0)
        return fail(GOFANN_ERR_INVALID, "exact_posting_scan: base and queries must be 16-byte aligned");
    if (routes->n_routes == 0) return GOFANN_OK;
    ScanArgs a{};
    a.routes = *routes;
    a.attrs = make_attr_view(attrs);
    if (!attrs) a.attrs.n_samples = n_samples;
    a.posting_ids = posting_ids;
    a.route_begin = route_begin;
    a.route_count = route_count;
    a.k = k;
    a.out_ids = out_ids;
    a.out_d = out_dists;
    a.base = base;
    a.queries = queries;
    a.dim = dim;
    a.row_bytes = dim * elem;
    const size_t smem = static_cast<size_t>(kSortSize) * 8 + static_cast<size_t>(kScanWarps) * kWarp * 8 + a.row_bytes;
    cudaStream_t s = as_stream(stream);
    if (dtype == GOFANN_DTYPE_U8) return launch_scan<kScanExactU8, 0>(a, smem, false, s, "posting_scan_kernel(exact u8)");
    if (dtype == GOFANN_DTYPE_F16)
        return launch_scan<kScanExactF16, 0>(a, smem, false, s, "posting_scan_kernel(exact f16)");
    return launch_scan<kScanExactF32, 0>(a, smem, false, s, "posting_scan_kernel(exact f32)");
}

int gofann_segment_merge(const uint32_t* seg_indptr, uint32_t n_routes, const uint32_t* seg_ids,
                         const float* seg_dists, int32_t shortlist_k, uint32_t* out_ids, float* out_dists,
                         void* stream)
{
    if (!seg_indptr || !seg_ids || !seg_dists || !out_ids || !out_dists)
        return fail(GOFANN_ERR_INVALID, "segment_merge: null argument");
    if (shortlist_k < 1 || shortlist_k > GOFANN_MAX_SHORTLIST)
        return fail(GOFANN_ERR_INVALID, "segment_merge: shortlist %d outside 1..%d", shortlist_k,
                    GOFANN_MAX_SHORTLIST);
    if (n_routes == 0) return GOFANN_OK;
    const size_t smem = static_cast<size_t>(kSortSize) * 8;
    const int sms = sm_count() > 0 ? sm_count() : 148;
    const unsigned blocks = n_routes < static_cast<uint32_t>(sms) * 8 ? n_routes : static_cast<unsigned>(sms) * 8;
    segment_merge_kernel<<<blocks, kScanThreads, smem, as_stream(stream)>>>(seg_indptr, n_routes, seg_ids, seg_dists,
                                                                           shortlist_k, out_ids, out_dists);
    GOFANN_CHECK_LAUNCH("segment_merge_kernel");
    return GOFANN_OK;
}

}  // extern "C"
