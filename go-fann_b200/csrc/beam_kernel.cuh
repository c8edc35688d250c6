// beam_kernel.cuh — the persistent filtered graph beam-search kernel (one
// warp per route), shared by the files that instantiate its variants
// (beam_variants_*.cu) and by the host entry points (beam_search.cu).
//
// Semantics follow the device-resident traversal loop of the reference,
// run_pq_search_one_block (src/search/pq/backend_pq.cu:3988-5013) with
// cooperative pickup, and its RaBitQ twin run_rabitq_search_one_block
// (src/search/rabitq/backend_rabitq.cu:3496-4292): symmetric min-max
// frontier of queue_size+1 entries, 4096-slot visited hash, stop top-k with
// fixed/adaptive early stop, binary-heap result shortlist, DNF predicate with
// the alpha penalty.  Every decision that fixes which ids come back (pickup
// order, frontier admission/eviction, heap layouts, hash insertion order) is
// kept identical; the B200 kernel parallelises the rest across the warp:
//   * neighbour rows are read by 32 lanes at once and visited-tested in
//     parallel (the reference tests all neighbours before any insertion of
//     the same step, so a parallel test is exact), compacted in order by
//     ballot/popc;
//   * each lane scores whole candidates: the PQ ADC replays the reference's
//     lane-strided partials and xor butterfly inside one thread, so 32
//     candidates are scored in one dependent round instead of 32;
//   * predicate pass bits and the frontier-threshold rejections are computed
//     by all lanes; lane 0 only runs the surviving min-max heap insertions,
//     which are order dependent.
// Warps are persistent: each pulls route indices from a device counter.
#pragma once

#include "pq_device.cuh"
#include "rq_device.cuh"

namespace gofann {
namespace beam {

constexpr int kWarpsPerBlock = 4;
// GOFANN_PQ_U8 blocks share one packed codebook in shared memory: one large
// block per SM (48 KB codebook + 24 warps' areas) amortises it.
constexpr int kU8BlockWarps = 24;
constexpr int kMaxBlockWarps = 32;  // scratch sizing bound over all variants

template <int kMode>
constexpr int block_warps() { return kMode == GOFANN_PQ_U8 ? kU8BlockWarps : kWarpsPerBlock; }
// Blocks per SM the register budget is sized for: 24 warps where registers
// bound the occupancy; with the table in shared memory one block fits anyway.
template <int kMode>
constexpr int min_blocks() { return kMode == GOFANN_PQ_U8 ? 1 : (kMode == GOFANN_PQ_LUT_SHARED ? 1 : 6); }
// Frontier payload: local row in bits 0..29, bit 31 = expanded ("used",
// backend_pq.cu:738-758), bit 30 = the row passed the route's DNF predicate
// when it was admitted (recorded only with predicate bias, where the
// predicate is evaluated at admission; the expansion then reuses it instead
// of evaluating the same predicate on the same sample again).
constexpr uint32_t kPassBit = 0x40000000u;
constexpr uint32_t kRowMask = 0x3fffffffu;
constexpr int kMaxSteps = 1 << 22;  // hard bound when max_steps == 0

struct WarpState {
    FPair now, next;
    int heap_size, stop_size, topk_size, finished;
    int exhausted, expanded, passed, len;
    float stop_worst, penalty, maxv;
    int brk, nfr, reject_all;
    uint32_t n_dist, n_probe, n_admit;
    uint32_t rej[2];
    uint32_t pass[2];
    uint32_t adm[2];     // candidates admitted to the frontier this step
    int hash_count;      // values in the visited table
    int serial_hash;     // 1: this step's insertions could fill the table
};

struct BeamArgs {
    gofann_graph graph;
    AttrView attrs;
    gofann_codes codes;
    gofann_prepared prep;
    gofann_routes routes;
    gofann_search_params p;
    gofann_search_out out;
    uint32_t* hash;          // [total_warps][4096]
    uint32_t* route_counter; // one uint32, zeroed before launch
    int32_t* status;
    uint32_t warp_smem;      // bytes of dynamic shared memory per warp
    uint32_t block_smem;     // bytes shared by the block ahead of the warps' areas
};

struct SmemLayout {
    uint32_t frontier, topk, stop, list, dist, prio, cbucket, cfree, state, table, total;
};

__host__ __device__ inline uint32_t align16(uint32_t x) { return (x + 15u) & ~15u; }

__host__ __device__ inline SmemLayout smem_layout(const gofann_search_params& p, const gofann_codes& c,
                                                  int pq_mode, uint32_t dim)
{
    SmemLayout s;
    uint32_t o = 0;
    // frontier: the reference heap, queue_size + 3 entries of 16 bytes
    s.frontier = o; o = align16(o + (p.queue_size + 3) * 12);
    s.topk = o; o = align16(o + (p.result_width + 1) * sizeof(RPair));
    s.stop = o; o = align16(o + (GOFANN_MAX_TOPK + 2) * sizeof(SPair));
    s.list = o; o = align16(o + GOFANN_MAX_DEGREE * 4);
    s.dist = o; o = align16(o + GOFANN_MAX_DEGREE * 4);
    s.prio = o; o = align16(o + GOFANN_MAX_DEGREE * 4);
    s.cbucket = o; o = align16(o + GOFANN_MAX_DEGREE * 4);
    s.cfree = o; o = align16(o + GOFANN_MAX_DEGREE * 4);
    s.state = o; o = align16(o + sizeof(WarpState));
    s.table = o;
    if (p.scorer == GOFANN_SCORER_PQ) {
        if (pq_mode == GOFANN_PQ_LUT_SHARED) o = align16(o + c.pq_dim * GOFANN_PQ_CENTROIDS * 4);
        if (pq_mode == GOFANN_PQ_DIRECT) o = align16(o + dim * 4);
        if (pq_mode == GOFANN_PQ_U8) o = align16(o + dim);  // query bytes
    } else {
        o = align16(o + 8 * (c.padded_dim / 32) * 4);
    }
    s.total = o;
    return s;
}

__device__ __forceinline__ int adaptive_limit(int queue_limit, int expanded, int pass, int stop_width)
{
    // adaptive_early_stop_limit, backend_pq.cu:2822-2854
    const int queue_base = queue_limit > 1 ? queue_limit : 1;
    int base_limit = (queue_base + 1) / 2;
    const int min_base = stop_width > 0 ? stop_width * 2 : 1;
    base_limit = base_limit > min_base ? base_limit : min_base;
    const int denom = (expanded + 16) > 1 ? (expanded + 16) : 1;
    const int pw = pass + 8;
    const int pest = pw < denom ? pw : denom;
    const int rej = (denom - pest) > 0 ? (denom - pest) : 0;
    const int64_t num = static_cast<int64_t>(queue_limit) * rej;
    int extra = static_cast<int>((num + (2 * denom - 1)) / (2 * denom));
    extra = extra > 0 ? extra : 0;
    extra = extra < 32 ? extra : 32;
    return base_limit + extra;
}

__device__ __forceinline__ bool stop_now(const gofann_search_params& p, const WarpState& st, int step)
{
    bool es = false;
    if (p.early_stop_mode == GOFANN_EARLY_STOP_ADAPTIVE)
        es = st.finished >= adaptive_limit(p.queue_size, st.expanded, st.passed, p.stop_width);
    else if (p.early_stop_mode == GOFANN_EARLY_STOP_FIXED)
        es = st.finished >= p.finish_limit;
    const int cap = p.max_steps > 0 ? p.max_steps : kMaxSteps;
    return st.exhausted || es || step >= cap;
}

// Adjacency row of local row `row`: ids of neighbours lane and lane + 32 in
// registers (UINT32_MAX past the degree).  The node expanded next is fixed
// one step ahead (the reference picks `next` before processing `now`,
// backend_pq.cu:4257-4278), so its row is loaded while the current step
// scores and admits candidates.
__device__ __forceinline__ void load_row_ids(uint32_t (&ids)[GOFANN_MAX_DEGREE / kWarp], const uint32_t* adjacency,
                                             uint32_t label_offset, uint32_t degree, uint32_t deg, uint32_t row,
                                             int lane, uint64_t pol)
{
    const uint32_t* src = adjacency + static_cast<size_t>(label_offset + row) * degree;
#pragma unroll
    for (int h = 0; h < GOFANN_MAX_DEGREE / kWarp; ++h) {
        const uint32_t i = h * kWarp + lane;
        ids[h] = i < deg ? ldg_u32(src + i, pol) : kU32Max;
    }
}

__device__ __forceinline__ uint32_t ordered_bits(float f)
{
    if (f == 0.0f) f = 0.0f;
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// kMode: PQ_LUT_GLOBAL / PQ_LUT_SHARED read a table row; PQ_DIRECT evaluates
// entries from the query row (shared memory) and the codebook; kW is the
// subvector width when it is 4 (vector loads), else 0; kMaxM bounds pq_dim.
template <int kScorer, int kMode, int kW, int kMaxM>
struct Scorer {
    const float* lut_row;  // PQ table row, or the query row in PQ_DIRECT
    const float* cent;     // PQ_DIRECT codebook
    int dim;
    RqQueryView rq;        // RaBitQ
    uint64_t keep, stream; // L2 policies: per-route tables / streaming rows
    const uint32_t* qw;    // PQ_U8: query words (shared memory)
    const uint32_t* cbw;   // PQ_U8: packed codebook (shared memory)
    int wq;                // PQ_U8: words per subvector
    __device__ __forceinline__ float operator()(const gofann_codes& c, uint32_t sample) const
    {
        if constexpr (kScorer == GOFANN_SCORER_PQ)
            return code_row(c, c.pq_codes + static_cast<size_t>(sample) * c.pq_dim);
        else
            return rq_estimate(c, rq, sample);
    }
    // PQ distance of the code row at `code` (the codes array or a row record)
    __device__ __forceinline__ float code_row(const gofann_codes& c, const uint8_t* code) const
    {
        if constexpr (kScorer == GOFANN_SCORER_PQ) {
            if constexpr (kMode == GOFANN_PQ_DIRECT) {
                return pq_adc_direct<kW, kMaxM>(lut_row, cent, dim, code, static_cast<int>(c.pq_dim), keep, stream);
            } else if constexpr (kMode == GOFANN_PQ_U8) {
                if constexpr (kW == 4) {  // 4-wide subvectors, pq_dim a multiple of 16 (host-checked)
                    return pq_adc_u8_chunked(qw, cbw, code, static_cast<int>(c.pq_dim), stream);
                } else {
                    uint32_t cw[kMaxM / 4];
                    load_code_words<kMaxM>(code, static_cast<int>(c.pq_dim), cw, stream);
                    return pq_adc_u8<kMaxM>(qw, cbw, cw, static_cast<int>(c.pq_dim), wq);
                }
            } else {
                uint32_t cw[kMaxM / 4];
                load_code_words<kMaxM>(code, static_cast<int>(c.pq_dim), cw, stream);
                if constexpr (kMode == GOFANN_PQ_LUT_GLOBAL)
                    return pq_adc_words_global<kMaxM>(lut_row, cw, static_cast<int>(c.pq_dim), keep);
                else
                    return pq_adc_words<kMaxM>(lut_row, cw, static_cast<int>(c.pq_dim));
            }
        } else {
            return 0.0f;  // RaBitQ scores by sample (operator())
        }
    }
};

// Cooperative pickup (backend_pq.cu:844-893; RaBitQ backend_rabitq.cu:
// 924-970): lane l scans entries l+1, l+33, ... keeping its first unused
// entry of smallest key, then a shfl_down tree merges lane l+off into lane l
// for off = 16..1.  In the reference as compiled for sm_100a a merge replaces
// the receiving lane's candidate only by a strictly smaller key (run on a
// B200 on tie-heavy frontiers: the source's equal-key index tie-break never
// takes effect), so among lanes holding the minimum the tree's merge order
// decides: lane 0 absorbs lanes 16, 8, 24, 4, 20, ... -- the order of the
// 5-bit-reversed lane index.  The pick is therefore the minimum of (key,
// bit-reversed lane, position within the lane), found here with two warp
// min-reductions; keys compare by their order-preserving bit pattern (equal
// to float order for the non-NaN keys a frontier holds, -0 folded onto +0).
__device__ __forceinline__ bool smmh_pickup(const Smmh& h, int size, FPair* out, int lane)
{
    uint32_t best = kU32Max, pos = 0;
    int k = 0;
    for (int i = lane + 1; i < size; i += kWarp, ++k) {
        if (h.val[i] & kPoolUsed) continue;
        const uint32_t kb = ordered_bits(h.key[i]);
        if (kb < best) {
            best = kb;
            pos = static_cast<uint32_t>(k);
        }
    }
    const uint32_t m = __reduce_min_sync(kFull, best);
    const uint32_t rank = best == m && m != kU32Max ? ((__brev(static_cast<uint32_t>(lane)) >> 27) << 16) | pos
                                                    : kU32Max;
    const uint32_t w = __reduce_min_sync(kFull, rank);
    const int bi = w == kU32Max ? -1 : static_cast<int>((__brev(w >> 16) >> 27) + 1 + kWarp * (w & 0xffffu));
    if (lane == 0 && bi >= 0) {
        out->first = h.key[bi];
        out->second = h.val[bi];
        out->base = h.base[bi];
        h.val[bi] |= kPoolUsed;
    }
    __syncwarp();
    return bi >= 0;
}

// Smallest key (or unbiased score) over the unused entries: fminf is exact
// and order-independent for the non-NaN values a frontier holds.
__device__ __forceinline__ float smmh_unused_min(const Smmh& h, int size, bool use_base, int lane)
{
    float m = FLT_MAX;
    for (int i = lane + 1; i < size; i += kWarp)
        if (!(h.val[i] & kPoolUsed)) m = fminf(m, use_base ? h.base[i] : h.key[i]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fminf(m, __shfl_xor_sync(kFull, m, off));
    return m;
}

// Per-warp shared-memory views.
struct WarpBufs {
    Smmh heap;          // frontier: the reference's min-max heap
    RPair* topk;
    SPair* stopk;
    uint32_t* list;
    float* dist;
    float* prio;
    uint32_t* cbucket;  // per listed candidate: the bucket its test ended in
    uint32_t* cfree;    // ... and that bucket's free-slot mask
    WarpState* st;
    uint32_t* hash;
};

// One route from its seed to its shortlist.
template <int kScorer, bool kBias, int kMode, int kW, int kMaxM, bool kExt>
__device__ __forceinline__ void run_route(const BeamArgs& a, const WarpBufs& w,
                                          const Scorer<kScorer, kMode, kW, kMaxM>& score, uint32_t route,
                                          uint32_t label_offset, uint32_t begin_id, uint64_t qbit, bool pred_on,
                                          uint32_t deg, uint64_t stream, int lane)
{
    const gofann_search_params& p = a.p;
    const int QS = p.queue_size, SW = p.stop_width, RW = p.result_width;
    const uint32_t meta_off = GOFANN_RECORD_META(a.codes.pq_dim);
    WarpState& st = *w.st;
    const Smmh& h = w.heap;
    RPair* topk = w.topk;
    SPair* stopk = w.stopk;
    uint32_t* list = w.list;
    float* dist = w.dist;
    float* prio = w.prio;
    uint32_t* hash = w.hash;

    // signature bits every passing record carries: those of the labels of a
    // route whose predicate is one clause without range atoms (a record's
    // signature holds the bit of each label of its row)
    uint32_t sig_need = 0;
    if (kBias && pred_on && a.graph.records != nullptr) {
        const uint32_t c0 = a.routes.pred_offsets[route];
        if (a.routes.pred_offsets[route + 1] == c0 + 1) {
            const gofann_clause c = a.routes.clauses[c0];
            if (c.range_begin == c.range_end)
                for (uint32_t j = c.label_begin; j < c.label_end; ++j)
                    sig_need |= GOFANN_LABEL_SIG_BIT(a.routes.pred_handles[j]);
        }
    }

    // visited table clear (native_visited_hash::clear)
    {
        uint4* h4 = reinterpret_cast<uint4*>(hash);
        const uint4 e = make_uint4(kU32Max, kU32Max, kU32Max, kU32Max);
        for (int i = lane; i < kHashCap / 4; i += kWarp) h4[i] = e;
    }
    __syncwarp();

    // start node (backend_pq.cu:4172-4209)
    if (lane == 0) {
        const uint32_t begin_sample = a.graph.row_to_sample[label_offset + begin_id];
        const float start = score(a.codes, begin_sample);
        float penalty = 0.0f;
        if (kBias) {
            const double wide = static_cast<double>(p.alpha) * fmax(static_cast<double>(fabsf(start)), 1e-6);
            penalty = isfinite(wide) ? static_cast<float>(fmin(wide, static_cast<double>(FLT_MAX))) : 0.0f;
        }
        st.penalty = penalty;
        st.heap_size = 1;
        st.stop_size = 0;
        st.topk_size = 0;
        st.stop_worst = -FLT_MAX;
        st.finished = 0;
        st.exhausted = 0;
        st.expanded = 0;
        st.passed = 0;
        st.n_dist = 1;
        st.n_probe = 0;
        st.n_admit = 0;
        FPair kp;
        kp.first = start;
        kp.second = begin_id;
        kp.base = start;
        if (kBias && pred_on && pred_matches<kExt>(a.routes, a.attrs, route, begin_sample)) kp.second |= kPassBit;
        h.key[1] = kp.first; h.val[1] = kp.second; h.base[1] = kp.base;
        st.heap_size = 2;
        hash_add(hash, begin_id);
        st.hash_count = 1;
    }
    __syncwarp();
    smmh_pickup(h, st.heap_size, &st.now, lane);
    // adjacency ids of the node expanded now and of the one expanded next
    uint32_t nb[GOFANN_MAX_DEGREE / kWarp], nb_next[GOFANN_MAX_DEGREE / kWarp];
#pragma unroll
    for (int h = 0; h < GOFANN_MAX_DEGREE / kWarp; ++h) nb_next[h] = kU32Max;
    load_row_ids(nb, a.graph.adjacency, label_offset, a.graph.degree, deg, st.now.second & kRowMask, lane, stream);

    int step = 0;
    for (;;) {
        if (step != 0 && st.heap_size <= 1) break;
        ++step;
        if (step != 1) {
            FPair nx;
            const bool found = smmh_pickup(h, st.heap_size, &st.next, lane);
            float unused_min = FLT_MAX;
            if (found && st.stop_size == SW && p.pending_base_stop && pred_on)
                unused_min = smmh_unused_min(h, st.heap_size, kBias, lane);
            if (lane == 0) {
                if (!found) {
                    st.exhausted = 1;
                    nx.first = FLT_MAX; nx.second = kU32Max; nx.base = FLT_MAX;
                    st.next = nx;
                } else if (st.stop_size == SW) {
                    float pending = st.next.first;
                    if (p.pending_base_stop && pred_on) {
                        float m = fminf(FLT_MAX, kBias ? st.now.base : st.now.first);
                        m = fminf(m, kBias ? st.next.base : st.next.first);
                        pending = fminf(m, unused_min);
                    }
                    if (p.early_stop_mode != GOFANN_EARLY_STOP_OFF && st.stop_worst <= pending) ++st.finished;
                }
            }
            __syncwarp();
            if (found)
                load_row_ids(nb_next, a.graph.adjacency, label_offset, a.graph.degree, deg,
                             st.next.second & kRowMask, lane, stream);
        }
        if (st.exhausted) break;
        const uint32_t now_row = st.now.second & kRowMask;
        const uint32_t grow = label_offset + now_row;

        if (lane == 0) {
            // filter verdict of the expanded node (backend_pq.cu:4394-4440)
            const bool bit_match = a.graph.row_filter_mask ? (a.graph.row_filter_mask[grow] & qbit) != 0ull
                                                           : qbit != 0ull;
            const bool need_sample = a.routes.range_modes != nullptr || p.full_label_check != 0 ||
                                     (pred_on && !kBias);
            const uint32_t sample = need_sample ? a.graph.row_to_sample[grow] : 0u;
            uint32_t active = 0, matched = 0;
            if (a.routes.range_modes) {
                for (uint32_t i = 0; i < a.routes.range_count; ++i) {
                    const size_t qf = static_cast<size_t>(route) * a.routes.range_count + i;
                    const uint8_t mode = a.routes.range_modes[qf];
                    if (mode == 0) continue;
                    ++active;
                    if (a.routes.range_lower && a.routes.range_upper && a.attrs.ranges &&
                        range_match(mode, a.routes.range_lower[qf], a.routes.range_upper[qf],
                                    a.attrs.ranges[static_cast<size_t>(sample) * a.routes.range_count + i]))
                        ++matched;
                }
                if (!a.routes.range_lower || !a.routes.range_upper || !a.attrs.ranges) matched = 0;
            }
            const bool exact_range = active == 0 || matched == active;
            int nfr = (p.full_label_check == 0 || labels_match(a.routes, a.attrs, route, sample)) ? 1 : 2;
            if (pred_on) {
                if (kBias)
                    nfr = (st.now.second & kPassBit) ? 1 : 2;
                else
                    nfr = pred_matches<kExt>(a.routes, a.attrs, route, sample) ? 1 : 2;
                ++st.n_probe;
            } else if (!a.routes.route_compiled || !a.routes.route_compiled[route]) {
                nfr = (nfr == 1 && bit_match && exact_range) ? 1 : 2;
            }
            st.nfr = nfr;
            st.brk = stop_now(p, st, step) ? 1 : 0;
            if (!st.brk) {
                if (a.out.trace && static_cast<uint32_t>(st.expanded) < a.out.trace_width)
                    a.out.trace[static_cast<size_t>(route) * a.out.trace_width + st.expanded] = now_row;
                ++st.expanded;
                if (nfr == 1) {
                    // stop top-k and result heap (backend_pq.cu:4583-4630)
                    ++st.passed;
                    const float current = kBias ? st.now.base : st.now.first;
                    RPair te;
                    te.first = current;
                    te.second = now_row;
                    SPair se;
                    se.first = current;
                    se.pad = 0;
                    se.second = (static_cast<uint64_t>(__float_as_uint(current)) << 32) | now_row;
                    bool improved = false;
                    if (st.stop_size < SW) {
                        stopk[st.stop_size++] = se;
                        bheap_push(stopk, st.stop_size);
                        improved = true;
                        if (st.stop_size == 1 || current > st.stop_worst) st.stop_worst = current;
                    } else if (se.first < stopk[0].first) {
                        stopk[st.stop_size++] = se;
                        bheap_push(stopk, st.stop_size);
                        const SPair removed = bheap_pop(stopk, st.stop_size);
                        --st.stop_size;
                        improved = true;
                        const uint32_t removed_bits = static_cast<uint32_t>(removed.second >> 32);
                        if (current > st.stop_worst) {
                            st.stop_worst = current;
                        } else if (removed_bits == __float_as_uint(st.stop_worst)) {
                            st.stop_worst = -FLT_MAX;
                            for (int i = 0; i < st.stop_size; ++i) {
                                const float pd = __uint_as_float(static_cast<uint32_t>(stopk[i].second >> 32));
                                if (pd > st.stop_worst) st.stop_worst = pd;
                            }
                        }
                    }
                    if (p.early_stop_mode == GOFANN_EARLY_STOP_ADAPTIVE && improved) st.finished = 0;
                    if (st.topk_size < RW) {
                        topk[st.topk_size++] = te;
                        bheap_push(topk, st.topk_size);
                    } else if (te.first < topk[0].first) {
                        topk[st.topk_size++] = te;
                        bheap_push(topk, st.topk_size);
                        bheap_pop(topk, st.topk_size);
                        --st.topk_size;
                    }
                }
            }
        }
        __syncwarp();
        if (st.brk) break;

        // neighbour list: visited test of the row's ids (in registers), in-order
        // compaction
        int len = 0;
#pragma unroll
        for (int half = 0; half < GOFANN_MAX_DEGREE / kWarp; ++half) {
            const uint32_t idx = nb[half];
            BucketProbe pr{kU32Max, 0u, true};
            if (idx != kU32Max) pr = bucket_probe(hash, idx);
            const bool keep = !pr.found;
            const unsigned m = __ballot_sync(kFull, keep);
            if (keep) {
                const int pos = len + __popc(m & ((1u << lane) - 1u));
                list[pos] = idx;
                w.cbucket[pos] = pr.bucket;
                w.cfree[pos] = pr.free_mask;
            }
            len += __popc(m);
        }
        __syncwarp();
        if (lane == 0) {
            st.len = len;
            st.brk = stop_now(p, st, step) ? 1 : 0;
        }
        __syncwarp();
        if (st.brk) break;

        // score and predicate of every listed candidate, one candidate per
        // lane (from its row record when the graph has them: the code row and
        // the label-row range share one line, and the label read overlaps the
        // distance arithmetic); priorities, pass bits and the candidates
        // certainly rejected (above the heap maximum while the heap is full:
        // the maximum only decreases within a step) as ballots
        const bool use_rec = kScorer == GOFANN_SCORER_PQ && a.graph.records != nullptr;
        const bool full = st.heap_size >= QS + 1;
        const float maxv = full ? h.key[2] : 0.0f;
#pragma unroll 1
        for (int half = 0; half < (len + kWarp - 1) / kWarp; ++half) {
            const int i = half * kWarp + lane;
            bool reject = false, pass = false;
            if (i < len) {
                float d;
                if (use_rec) {
                    const uint8_t* rec =
                        a.graph.records + static_cast<size_t>(label_offset + list[i]) * a.graph.record_stride;
                    const uint4 meta = ldg_u32x4(reinterpret_cast<const uint4*>(rec + meta_off), stream);
                    if (kBias && pred_on && (meta.w & sig_need) == sig_need) {
                        // the label row from the record when it is stored there
                        const bool inl = meta.z <= GOFANN_RECORD_INLINE_LABELS;
                        const uint32_t* lab = inl ? reinterpret_cast<const uint32_t*>(rec + meta_off + 16)
                                                  : a.attrs.indices;
                        const uint64_t lb = inl ? 0ull : meta.y;
                        pass = pred_matches_row<kExt>(a.routes, a.attrs, route, meta.x, lab, lb, lb + meta.z);
                    }
                    d = score.code_row(a.codes, rec);
                } else {
                    const uint32_t smp = ldg_u32(a.graph.row_to_sample + label_offset + list[i], stream);
                    if (kBias && pred_on) pass = pred_matches<kExt>(a.routes, a.attrs, route, smp);
                    d = score(a.codes, smp);
                }
                const float pr = (kBias && pred_on) ? pred_priority(d, st.penalty, pass) : d;
                dist[i] = d;
                prio[i] = pr;
                reject = full && maxv < pr;
            }
            const unsigned rm = __ballot_sync(kFull, reject);
            const unsigned pm = __ballot_sync(kFull, pass);
            if (lane == 0) {
                st.rej[half] = rm;
                st.pass[half] = pm;
            }
        }
        __syncwarp();
        const uint32_t rej[2] = {st.rej[0], len > kWarp ? st.rej[1] : 0u};
        const uint32_t pbits[2] = {st.pass[0], len > kWarp ? st.pass[1] : 0u};
        // frontier admissions in list order (order dependent), the whole warp
        // on each insert / pop_max; the visited-table insertions of the
        // admitted rows follow, concurrently when the table cannot fill
        {
            int hs = st.heap_size;
            uint32_t adm[2] = {0u, 0u};
            int n_adm = 0;
#pragma unroll
            for (int half = 0; half < GOFANN_MAX_DEGREE / kWarp; ++half) {
                // the candidates not rejected up front, in list order
                const int n_here = len - half * kWarp;
                unsigned todo = n_here <= 0 ? 0u : ~rej[half] & (n_here >= kWarp ? kFull : (1u << n_here) - 1u);
                while (todo) {
                    const int i = half * kWarp + __ffs(todo) - 1;
                    todo &= todo - 1;
                    const float key = prio[i];
                    if (hs >= QS + 1 && h.key[2] < key) continue;
                    const uint32_t val = list[i] | (((pbits[half] >> (i & 31)) & 1u) ? kPassBit : 0u);
                    smmh_insert_warp(h, hs, key, val, dist[i], lane);
                    ++hs;
                    adm[half] |= 1u << (i & 31);
                    ++n_adm;
                    if (hs >= QS + 2) {
                        smmh_pop_max_warp(h, hs, lane);
                        --hs;
                    }
                }
            }
            if (lane == 0) {
                st.heap_size = hs;
                st.n_dist += static_cast<uint32_t>(len);
                if (kBias && pred_on) st.n_probe += static_cast<uint32_t>(len);
                st.n_admit += static_cast<uint32_t>(n_adm);
                st.adm[0] = adm[0];
                st.adm[1] = adm[1];
                // admitted rows are absent from the table (they passed the
                // visited test this step); the reference inserts them right
                // after each admission, nothing reads the table before the
                // next step, so deferring the inserts is exact
                st.serial_hash = st.hash_count + n_adm > kHashCap ? 1 : 0;
            }
            __syncwarp();
        }
        {
            // Each admitted row takes the free slot its test saw, ranked among
            // the admitted rows whose tests ended in the same bucket (nothing
            // else wrote the table since): plain stores; a bucket that runs
            // out sends the rest to the atomic walk, after the stores.  When
            // the table could fill during the step, or an adjacency row lists
            // an id twice (both copies are admitted, as in the reference, but
            // its second insert is a no-op; equal ids end their tests in the
            // same bucket, so the rank scan sees the repeat), lane 0 inserts
            // one by one in list order instead.
            const uint32_t adm0 = st.adm[0], adm1 = st.adm[1];
            int slot[GOFANN_MAX_DEGREE / kWarp] = {-1, -1};
            bool serial = st.serial_hash != 0;
            if (!serial) {
                bool repeat = false;
#pragma unroll
                for (int half = 0; half < GOFANN_MAX_DEGREE / kWarp; ++half) {
                    const int i = half * kWarp + lane;
                    if (((half == 0 ? adm0 : adm1) >> lane) & 1u) {
                        const uint32_t b = w.cbucket[i];
                        int rank = 0;
#pragma unroll
                        for (int h2 = 0; h2 < GOFANN_MAX_DEGREE / kWarp; ++h2) {
                            uint32_t before = h2 == 0 ? adm0 : adm1;
                            if (h2 > half) before = 0u;
                            else if (h2 == half) before &= (1u << lane) - 1u;
                            while (before) {
                                const int j = h2 * kWarp + __ffs(before) - 1;
                                before &= before - 1;
                                if (w.cbucket[j] == b) {
                                    ++rank;
                                    repeat |= list[j] == list[i];
                                }
                            }
                        }
                        const int sl = nth_set_bit(w.cfree[i], rank);
                        slot[half] = sl >= 0 ? sl : -2;  // -2: bucket ran out, atomic walk
                    }
                }
                serial = __any_sync(kFull, repeat);
            }
            if (serial) {
                if (lane == 0) {
                    int added = 0;
                    for (int i = 0; i < len; ++i)
                        if (((i < kWarp ? adm0 : adm1) >> (i & 31)) & 1u) added += hash_add(hash, list[i]) ? 1 : 0;
                    st.hash_count += added;
                }
            } else {
                if (lane == 0) st.hash_count += __popc(adm0) + __popc(adm1);
#pragma unroll
                for (int half = 0; half < GOFANN_MAX_DEGREE / kWarp; ++half)
                    if (slot[half] >= 0)
                        hash[w.cbucket[half * kWarp + lane] * kBucketSlots + slot[half]] = list[half * kWarp + lane];
                __syncwarp();
#pragma unroll
                for (int half = 0; half < GOFANN_MAX_DEGREE / kWarp; ++half)
                    if (slot[half] == -2) hash_add_concurrent(hash, list[half * kWarp + lane]);
            }
        }
        __syncwarp();
        if (step == 1) {
            const bool found = smmh_pickup(h, st.heap_size, &st.next, lane);
            if (lane == 0 && !found) {
                st.exhausted = 1;
                FPair nx;
                nx.first = FLT_MAX; nx.second = kU32Max; nx.base = FLT_MAX;
                st.next = nx;
            }
            if (found)
                load_row_ids(nb_next, a.graph.adjacency, label_offset, a.graph.degree, deg,
                             st.next.second & kRowMask, lane, stream);
        }
        if (lane == 0) st.now = st.next;
        // the next step's visited-table lines (after this step's inserts),
        // fetched now into L1.  The neighbours' records are not prefetched:
        // the prefetch would also fetch the records of visited neighbours,
        // which are never read.  On the 10M categorical workload a
        // one-step-ahead L2 prefetch of every neighbour's record made the
        // traversal 1.1 % slower (80.5 against 79.6 ms per batch) and added a
        // quarter to its DRAM reads; a 64-byte bulk prefetch was 10 % slower.
#pragma unroll
        for (int h = 0; h < GOFANN_MAX_DEGREE / kWarp; ++h) {
            nb[h] = nb_next[h];
            if (nb[h] != kU32Max && !st.exhausted) prefetch_l1(hash + home_bucket(nb[h]) * kBucketSlots);
        }
        __syncwarp();
    }

    // emit the shortlist ascending (in-place heap sort of the result heap)
    if (lane == 0) {
        const int valid = st.topk_size;
        for (int i = 0; i < valid; ++i) {
            const int n = valid - i;
            const RPair r = bheap_pop(topk, n);
            topk[n - 1] = r;
        }
        if (step >= (p.max_steps > 0 ? p.max_steps : kMaxSteps) && p.max_steps == 0 && a.status)
            atomicExch(a.status, GOFANN_ERR_CAPACITY);
    }
    __syncwarp();
    const int valid = st.topk_size;
    uint32_t* oid = a.out.ids + static_cast<size_t>(route) * RW;
    float* od = a.out.dists + static_cast<size_t>(route) * RW;
    for (int i = lane; i < RW; i += kWarp) {
        uint32_t id = kU32Max;
        float d = FLT_MAX;
        if (i < valid && topk[i].second != kU32Max) {
            id = a.graph.row_to_sample[label_offset + topk[i].second];
            d = topk[i].first;
        }
        oid[i] = id;
        od[i] = d;
    }
    if (a.out.trace)
        for (uint32_t i = static_cast<uint32_t>(st.expanded) + lane; i < a.out.trace_width; i += kWarp)
            a.out.trace[static_cast<size_t>(route) * a.out.trace_width + i] = kU32Max;
    if (lane == 0) {
        if (a.out.steps) a.out.steps[route] = step;
        if (a.out.counters) {
            uint32_t* c = a.out.counters + static_cast<size_t>(route) * 4;
            c[0] = static_cast<uint32_t>(st.expanded);
            c[1] = st.n_dist;
            c[2] = st.n_probe;
            c[3] = st.n_admit;
        }
    }
    __syncwarp();
}

template <int kScorer, bool kBias, int kMode, int kW, int kMaxM, bool kExt>
__global__ void __launch_bounds__(block_warps<kMode>() * 32, min_blocks<kMode>()) beam_search_kernel(BeamArgs a)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const gofann_search_params& p = a.p;
    const SmemLayout L = smem_layout(p, a.codes, kMode, a.prep.dim);
    if constexpr (kMode == GOFANN_PQ_U8) {
        // the block's packed codebook, checked while it is packed
        const bool ok = pack_u8_codebook(a.prep.pq_centroids, static_cast<int>(a.prep.dim),
                                         static_cast<int>(a.codes.pq_dim), reinterpret_cast<uint32_t*>(smem_raw),
                                         threadIdx.x, blockDim.x);
        if (__syncthreads_or(!ok)) {
            if (threadIdx.x == 0 && a.status) atomicExch(a.status, GOFANN_ERR_INVALID);
            return;
        }
    }
    unsigned char* base = smem_raw + a.block_smem + static_cast<size_t>(warp) * a.warp_smem;
    WarpBufs w;
    { const uint32_t fcap = static_cast<uint32_t>(p.queue_size) + 3;
    w.heap.key = reinterpret_cast<float*>(base + L.frontier);
    w.heap.val = reinterpret_cast<uint32_t*>(base + L.frontier + 4 * fcap);
    w.heap.base = reinterpret_cast<float*>(base + L.frontier + 8 * fcap); }
    w.topk = reinterpret_cast<RPair*>(base + L.topk);
    w.stopk = reinterpret_cast<SPair*>(base + L.stop);
    w.list = reinterpret_cast<uint32_t*>(base + L.list);
    w.dist = reinterpret_cast<float*>(base + L.dist);
    w.prio = reinterpret_cast<float*>(base + L.prio);
    w.cbucket = reinterpret_cast<uint32_t*>(base + L.cbucket);
    w.cfree = reinterpret_cast<uint32_t*>(base + L.cfree);
    w.st = reinterpret_cast<WarpState*>(base + L.state);
    float* table = reinterpret_cast<float*>(base + L.table);
    const uint32_t gwarp = blockIdx.x * (blockDim.x >> 5) + warp;
    w.hash = a.hash + static_cast<size_t>(gwarp) * kHashCap;
    const uint32_t deg = a.graph.degree < GOFANN_MAX_DEGREE ? a.graph.degree : GOFANN_MAX_DEGREE;
    const uint64_t keep = l2_keep_policy(), stream = l2_stream_policy();

    for (;;) {
        uint32_t route = 0;
        if (lane == 0) route = atomicAdd(a.route_counter, 1u);
        route = __shfl_sync(kFull, route, 0);
        if (route >= a.routes.n_routes) break;

        const uint32_t row = a.routes.query_row[route];
        const uint32_t label_offset = a.graph.label_offset[a.routes.group_id[route]];
        const uint32_t begin_id = a.routes.start_local[route];
        const uint64_t qbit = a.routes.filter_bits ? a.routes.filter_bits[route] : ~0ull;
        const bool pred_on = pred_enabled(a.routes, route);

        Scorer<kScorer, kMode, kW, kMaxM> score;
        score.keep = keep;
        score.stream = stream;
        if constexpr (kScorer == GOFANN_SCORER_PQ) {
            if constexpr (kMode == GOFANN_PQ_U8) {
                const int nw = static_cast<int>(a.prep.dim) / 4;
                const uint32_t* qr = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(a.prep.pq_query) +
                                                                       static_cast<size_t>(row) * a.prep.dim);
                uint32_t* qw = reinterpret_cast<uint32_t*>(table);
                for (int i = lane; i < nw; i += kWarp) qw[i] = qr[i];
                score.qw = qw;
                score.cbw = reinterpret_cast<const uint32_t*>(smem_raw);
                score.wq = static_cast<int>(a.prep.dim / a.codes.pq_dim) / 4;
            } else if constexpr (kMode == GOFANN_PQ_DIRECT) {
                const int dim = static_cast<int>(a.prep.dim);
                if (a.prep.pq_query_dtype == GOFANN_DTYPE_U8) {
                    const uint8_t* qr = static_cast<const uint8_t*>(a.prep.pq_query) + static_cast<size_t>(row) * dim;
                    for (int i = lane; i < dim; i += kWarp) table[i] = static_cast<float>(qr[i]);
                } else {
                    const float* qr = static_cast<const float*>(a.prep.pq_query) + static_cast<size_t>(row) * dim;
                    for (int i = lane; i < dim; i += kWarp) table[i] = qr[i];
                }
                score.lut_row = table;
                score.cent = a.prep.pq_centroids;
                score.dim = dim;
            } else {
                const float* g = a.prep.pq_lut + static_cast<size_t>(row) * a.codes.pq_dim * GOFANN_PQ_CENTROIDS;
                if constexpr (kMode == GOFANN_PQ_LUT_SHARED) {
                    const float4* s4 = reinterpret_cast<const float4*>(g);
                    float4* d4 = reinterpret_cast<float4*>(table);
                    const int n4 = static_cast<int>(a.codes.pq_dim) * GOFANN_PQ_CENTROIDS / 4;
                    for (int i = lane; i < n4; i += kWarp) d4[i] = __ldg(s4 + i);
                    score.lut_row = table;
                } else {
                    score.lut_row = g;
                }
            }
        } else {
            rq_build_planes(a.prep.rq_q8 + static_cast<size_t>(row) * a.codes.padded_dim,
                            static_cast<int>(a.codes.padded_dim), reinterpret_cast<uint32_t*>(table), lane,
                            kWarp);
            score.rq.planes = reinterpret_cast<const uint32_t*>(table);
            score.rq.scale = a.prep.rq_scale[row];
            score.rq.k1 = a.prep.rq_k1xsumq[row];
            score.rq.gdist = a.prep.rq_centroid_dist + static_cast<size_t>(row) * a.codes.num_anchors;
        }
        __syncwarp();

        run_route<kScorer, kBias, kMode, kW, kMaxM, kExt>(a, w, score, route, label_offset, begin_id, qbit, pred_on, deg,
                                                    stream, lane);
    }
}

using KernelFn = void (*)(BeamArgs);

// Variant pickers, one per file that instantiates them.  w4: 4-wide
// subvectors (vector loads / the chunked u8 scorer); small_m: pq_dim <= 64
// (a shorter unrolled subspace loop); ext: the routes' clauses may carry
// string and integer atoms.
KernelFn pick_u8(bool bias, bool w4, bool small_m, bool ext);
KernelFn pick_direct(bool bias, bool w4, bool small_m, bool ext);
KernelFn pick_table(bool shared, bool bias, bool small_m, bool ext);
KernelFn pick_rabitq(bool bias, bool ext);

}  // namespace beam
}  // namespace gofann
