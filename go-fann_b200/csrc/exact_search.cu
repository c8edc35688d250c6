// exact_search.cu — the Full-GPU exact-distance mode: filtered graph
// traversal scored by the exact L2 distance of the full base vectors held in
// HBM (no PQ or RaBitQ codes, no rerank), and the exact scan of posting
// lists.
//
// Semantics follow the reference's Full-GPU backend (putatio13/GO-FANN
// src/search/full_gpu/backend_full_gpu.cu):
//   run_full_gpu_highfreq_route  :1682-2043  (graph routes)
//   full_gpu_lowfreq_kernel      :2124-2260  (posting routes)
// Every decision that fixes which ids come back is kept: the symmetric
// min-max frontier of queue_size + 1 entries and its admission test (skip a
// candidate above the maximum of a full frontier), visited-table insertion of
// admitted rows only, pickup of the unused entry of smallest (distance,
// index), the expanded node's filter verdict (candidate_passes_device
// :1015-1092) and the sorted top-k of results with its duplicate rule
// (insert_best_result :1333-1375), and the stop rule: after every expansion
// but the first, the next node counts as a "finish hit" when the top-k is
// full and the next node's (distance, sample) does not beat its last entry,
// any other outcome resets the count (an improving expansion resets it in the
// adaptive mode), and the search stops when early_stop_reached (:133-151)
// says so.
//
// The reference runs one 128-thread block per route with lane 0 of each
// warp testing one neighbour and thread 0 doing all heap work.  Here one warp
// runs one route and warps are persistent (routes pulled from a device
// counter):
//   * the 64 neighbour ids are read and visited-tested by 32 lanes at once,
//     in the bucketed table layout of the traversal (same membership and
//     fill rule as the reference's 4,096-slot table), and compacted in edge
//     order by ballot;
//   * u8 distances: each lane computes whole candidates (16-byte row loads,
//     per-byte absolute differences and dp4a) -- an integer, order free;
//     f32 / f16: the warp computes candidates four at a time in the
//     reference's lane order and tree;
//   * the frontier is the min-max heap in struct-of-arrays form operated on
//     by the whole warp (smmh_insert_warp / smmh_pop_max_warp), with
//     candidates certainly above a full frontier's maximum rejected by one
//     ballot (the maximum of a full frontier never rises within a step);
//   * the top-k lives in registers (lane i holds entry i) and is updated
//     with ballots;
//   * the next node's adjacency row is loaded as soon as it is picked, and
//     the visited-table lines and row -> sample entries of its neighbours are
//     prefetched before the step ends.
#include "exact_device.cuh"

namespace gofann {
namespace exact {

constexpr int kBlockWarps = 4;
constexpr int kMaxSteps = 1 << 22;  // hard bound when max_steps == 0
constexpr size_t kCounterBytes = 256;

struct ExactArgs {
    gofann_graph graph;
    const uint32_t* label_size;  // [group_count] or null (derived from label_offset)
    AttrView attrs;
    gofann_routes routes;
    gofann_search_params p;
    gofann_search_out out;
    const void* base;
    const void* queries;
    uint32_t dim;
    uint32_t warp_smem;
    uint32_t* hash;
    uint32_t* route_counter;
    int32_t* status;
};

__host__ __device__ inline uint32_t align16(uint32_t x) { return (x + 15u) & ~15u; }

template <int kDtype>
constexpr uint32_t elem_bytes() { return kDtype == GOFANN_DTYPE_U8 ? 1u : (kDtype == GOFANN_DTYPE_F16 ? 2u : 4u); }

struct Layout {
    uint32_t key, val, base, list, dist, cbucket, cfree, query, total;
};
__host__ __device__ inline Layout layout(int queue_size, uint32_t dim, uint32_t elem)
{
    Layout L;
    const uint32_t fcap = static_cast<uint32_t>(queue_size) + 3;
    uint32_t o = 0;
    L.key = o; o = align16(o + fcap * 4);
    L.val = o; o = align16(o + fcap * 4);
    L.base = o; o = align16(o + fcap * 4);
    L.list = o; o = align16(o + GOFANN_MAX_DEGREE * 4);
    L.dist = o; o = align16(o + GOFANN_MAX_DEGREE * 4);
    L.cbucket = o; o = align16(o + GOFANN_MAX_DEGREE * 4);
    L.cfree = o; o = align16(o + GOFANN_MAX_DEGREE * 4);
    L.query = o; o = align16(o + dim * elem);
    L.total = o;
    return L;
}

// early_stop_reached / adaptive_early_stop_limit (backend_full_gpu.cu:
// 100-151) with stop_width = topk.
__device__ __forceinline__ bool early_stop_reached(int mode, int bad, int fixed, int queue, int expanded, int pass,
                                                   int stop_width)
{
    if (mode == GOFANN_EARLY_STOP_OFF) return false;
    if (mode == GOFANN_EARLY_STOP_ADAPTIVE) {
        const int queue_base = queue > 1 ? queue : 1;
        int base_limit = (queue_base + 1) / 2;
        const int min_base = stop_width > 0 ? stop_width * 2 : 1;
        base_limit = base_limit > min_base ? base_limit : min_base;
        const int denom = (expanded + 16) > 1 ? (expanded + 16) : 1;
        const int pw = pass + 8;
        const int pest = pw < denom ? pw : denom;
        const int rej = (denom - pest) > 0 ? (denom - pest) : 0;
        const int64_t num = static_cast<int64_t>(queue) * rej;
        int extra = static_cast<int>((num + (2 * denom - 1)) / (2 * denom));
        extra = extra > 0 ? extra : 0;
        extra = extra < 32 ? extra : 32;
        return bad >= base_limit + extra;
    }
    return bad >= fixed;
}

// better_result (backend_full_gpu.cu:1328-1331)
__device__ __forceinline__ bool better(float ld, uint32_t li, float rd, uint32_t ri)
{
    return ld < rd || (ld == rd && li < ri);
}

// The route's sorted top-k, lane i holding entry i (i < size).
struct TopK {
    float d;
    uint32_t id;
    int size;
};

// insert_best_result (backend_full_gpu.cu:1333-1375), warp-wide: an id
// already present keeps the smaller distance (a smaller one replaces it and
// moves); a full list takes the entry only if it beats the last one; the
// entry lands after every entry better than it.  Returns whether the list
// changed.
__device__ __forceinline__ bool topk_insert(TopK& t, int topk, float dist, uint32_t sample, int lane)
{
    bool changed = false;
    const unsigned dup = __ballot_sync(kFull, lane < t.size && t.id == sample);
    if (dup) {
        const int j = __ffs(dup) - 1;
        const float dj = __shfl_sync(kFull, t.d, j);
        if (!(dist < dj)) return false;
        // remove entry j: entries after it move up one place
        const float nd = __shfl_down_sync(kFull, t.d, 1);
        const uint32_t ni = __shfl_down_sync(kFull, t.id, 1);
        if (lane >= j && lane + 1 < t.size) { t.d = nd; t.id = ni; }
        --t.size;
        changed = true;
    }
    if (t.size == topk) {
        const float ld = __shfl_sync(kFull, t.d, topk - 1);
        const uint32_t li = __shfl_sync(kFull, t.id, topk - 1);
        if (!better(dist, sample, ld, li)) return changed;
    }
    const int pos = __popc(__ballot_sync(kFull, lane < t.size && better(t.d, t.id, dist, sample)));
    const float pd = __shfl_up_sync(kFull, t.d, 1);
    const uint32_t pi = __shfl_up_sync(kFull, t.id, 1);
    const int new_size = t.size < topk ? t.size + 1 : topk;
    if (lane > pos && lane < new_size) { t.d = pd; t.id = pi; }
    if (lane == pos) { t.d = dist; t.id = sample; }
    t.size = new_size;
    return true;
}

// candidate_passes_device (backend_full_gpu.cu:1015-1092): the route's
// filter bit against the row mask, then the residual labels (every query
// label but the route's own) and the active range atoms.
__device__ __forceinline__ bool candidate_passes(const ExactArgs& a, uint32_t route, uint64_t qbit, uint32_t grow,
                                                 uint32_t sample)
{
    const uint64_t mask = a.graph.row_filter_mask ? a.graph.row_filter_mask[grow] : ~0ull;
    if (qbit == 0ull || (mask & qbit) == 0ull) return false;
    const gofann_routes& r = a.routes;
    if (r.range_modes) {
        uint32_t active = 0, matched = 0;
        for (uint32_t i = 0; i < r.range_count; ++i) {
            const size_t qf = static_cast<size_t>(route) * r.range_count + i;
            const uint8_t mode = r.range_modes[qf];
            if (mode == 0) continue;
            ++active;
            if (r.range_lower && r.range_upper && a.attrs.ranges &&
                range_match(mode, r.range_lower[qf], r.range_upper[qf],
                            a.attrs.ranges[static_cast<size_t>(sample) * r.range_count + i]))
                ++matched;
        }
        if (active != 0 && (!a.attrs.ranges || matched != active)) return false;
    }
    return labels_match(r, a.attrs, route, sample);
}

// Frontier pickup: the unused entry of smallest (distance, index)
// (pickup_next_unused_from_pool_block, backend_full_gpu.cu:1536-1596).
// Lane l scans entries l+1, l+33, ... keeping its first minimum; two warp
// min-reductions pick the smallest distance, then the smallest index
// holding it.  Distances compare by their order-preserving bit pattern
// (non-negative here).
__device__ __forceinline__ int pickup(const Smmh& h, int size, int lane)
{
    uint32_t best = kU32Max, bi = kU32Max;
    for (int i = lane + 1; i < size; i += kWarp) {
        if (h.val[i] & kPoolUsed) continue;
        const uint32_t kb = __float_as_uint(h.key[i]) | 0x80000000u;
        if (kb < best) { best = kb; bi = static_cast<uint32_t>(i); }
    }
    const uint32_t m = __reduce_min_sync(kFull, best);
    const uint32_t w = __reduce_min_sync(kFull, best == m ? bi : kU32Max);
    return m == kU32Max ? -1 : static_cast<int>(w);
}

template <int kDtype>
__device__ __forceinline__ void run_route(const ExactArgs& a, unsigned char* wbase, uint32_t* hash, uint32_t route,
                                          int lane, uint64_t stream)
{
    const gofann_search_params& p = a.p;
    const int QS = p.queue_size, K = p.result_width;
    const Layout L = layout(QS, a.dim, elem_bytes<kDtype>());
    Smmh h;
    h.key = reinterpret_cast<float*>(wbase + L.key);
    h.val = reinterpret_cast<uint32_t*>(wbase + L.val);
    h.base = reinterpret_cast<float*>(wbase + L.base);
    uint32_t* list = reinterpret_cast<uint32_t*>(wbase + L.list);
    float* dist = reinterpret_cast<float*>(wbase + L.dist);
    uint32_t* cbucket = reinterpret_cast<uint32_t*>(wbase + L.cbucket);
    uint32_t* cfree = reinterpret_cast<uint32_t*>(wbase + L.cfree);
    unsigned char* q = wbase + L.query;
    const int n16 = static_cast<int>(a.dim / 16);

    TopK best{FLT_MAX, kU32Max, 0};
    int steps = 0, expanded = 0;
    uint32_t n_dist = 0, n_adm_total = 0;
    bool run = true;
    const uint32_t g = a.routes.group_id[route];
    uint32_t off = 0, gsize = 0, seed = kU32Max;
    if (g >= a.graph.group_count) {
        run = false;
    } else {
        off = a.graph.label_offset[g];
        gsize = a.label_size ? a.label_size[g]
                             : (g + 1 < a.graph.group_count ? a.graph.label_offset[g + 1] : a.graph.total_rows) - off;
        if (off > a.graph.total_rows || gsize > a.graph.total_rows - off) gsize = 0;
        seed = a.routes.start_local[route];
        if (gsize == 0 || seed >= gsize) run = false;
    }
    const uint32_t seed_sample = run ? a.graph.row_to_sample[off + seed] : kU32Max;
    if (seed_sample >= a.attrs.n_samples) run = false;

    if (run) {
        // query row to shared memory, visited table cleared
        const uint32_t row = a.routes.query_row[route];
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(a.queries) +
                                                          static_cast<size_t>(row) * a.dim * elem_bytes<kDtype>());
        const uint32_t n4 = (a.dim * elem_bytes<kDtype>()) / 16;
        for (uint32_t i = lane; i < n4; i += kWarp) reinterpret_cast<uint4*>(q)[i] = __ldg(src + i);
        uint4* h4 = reinterpret_cast<uint4*>(hash);
        const uint4 e = make_uint4(kU32Max, kU32Max, kU32Max, kU32Max);
        for (int i = lane; i < kHashCap / 4; i += kWarp) h4[i] = e;
        __syncwarp();
    }
    const uint64_t qbit = a.routes.filter_bits ? a.routes.filter_bits[route] : ~0ull;
    const size_t row_bytes = static_cast<size_t>(a.dim) * elem_bytes<kDtype>();
    const unsigned char* basep = static_cast<const unsigned char*>(a.base);

    int hs = 1, hash_count = 0;
    float now_key = 0.0f;
    uint32_t now_val = 0;
    if (run) {
        // seed (backend_full_gpu.cu:1818-1846)
        float sd;
        if constexpr (kDtype == GOFANN_DTYPE_U8) {
            const uint32_t v = l2_u8_thread(basep + static_cast<size_t>(seed_sample) * row_bytes,
                                            reinterpret_cast<const uint4*>(q), n16, stream);
            sd = static_cast<float>(v);
        } else {
            const void* rows[1] = {basep + static_cast<size_t>(seed_sample) * row_bytes};
            float o[1];
            l2_float_warp<kDtype, 1>(rows, q, static_cast<int>(a.dim), lane, stream, o);
            sd = o[0];
        }
        if (lane == 0) {
            h.key[1] = sd; h.val[1] = seed; h.base[1] = sd;
            hash_add(hash, seed);
        }
        hs = 2;
        hash_count = 1;
        n_dist = 1;
        __syncwarp();
        const int bi = pickup(h, hs, lane);
        now_key = h.key[bi];
        now_val = h.val[bi];
        __syncwarp();
        if (lane == 0) h.val[bi] |= kPoolUsed;
        __syncwarp();
    }

    const uint32_t deg = a.graph.degree < GOFANN_MAX_DEGREE ? a.graph.degree : GOFANN_MAX_DEGREE;
    uint32_t nb[2] = {kU32Max, kU32Max};
    if (run) {
        const uint32_t* src = a.graph.adjacency + static_cast<size_t>(off + (now_val & ~kPoolUsed)) * a.graph.degree;
        for (int hh = 0; hh < 2; ++hh) {
            const uint32_t i = hh * kWarp + lane;
            nb[hh] = i < deg ? ldg_u32(src + i, stream) : kU32Max;
        }
    }
    int passed = 0, fh = 0;
    bool first_step = true;
    const int cap = p.max_steps > 0 ? p.max_steps : kMaxSteps;
    while (run) {
        if (steps >= cap) {
            if (p.max_steps == 0 && lane == 0 && a.status) atomicExch(a.status, GOFANN_ERR_CAPACITY);
            break;
        }
        // expansion of `now`: filter verdict, top-k (backend_full_gpu.cu:1891-1922)
        const uint32_t now_local = now_val & ~kPoolUsed;
        const uint32_t now_row = off + now_local;
        const uint32_t now_sample = a.graph.row_to_sample[now_row];
        bool improved = false;
        if (a.out.trace && static_cast<uint32_t>(expanded) < a.out.trace_width && lane == 0)
            a.out.trace[static_cast<size_t>(route) * a.out.trace_width + expanded] = now_local;
        ++expanded;
        if (now_sample < a.attrs.n_samples && candidate_passes(a, route, qbit, now_row, now_sample)) {
            ++passed;
            improved = topk_insert(best, K, now_key, now_sample, lane);
        }
        ++steps;

        // neighbours: bounds, visited test, row -> sample; compacted in edge order
        int len = 0;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const uint32_t local = nb[hh];
            BucketProbe pr{kU32Max, 0u, true};
            uint32_t sample = kU32Max;
            if (local != kU32Max && local < gsize) {
                pr = bucket_probe(hash, local);
                if (!pr.found) {
                    sample = ldg_u32(a.graph.row_to_sample + off + local, stream);
                    if (sample >= a.attrs.n_samples) pr.found = true;
                }
            }
            const bool keep = !pr.found;
            const unsigned m = __ballot_sync(kFull, keep);
            if (keep) {
                const int pos = len + __popc(m & ((1u << lane) - 1u));
                list[pos] = local;
                cbucket[pos] = pr.bucket;
                cfree[pos] = pr.free_mask;
                dist[pos] = __uint_as_float(sample);  // sample id, replaced by the distance below
            }
            len += __popc(m);
        }
        __syncwarp();
        n_dist += static_cast<uint32_t>(len);

        // exact distances of the listed candidates
        if constexpr (kDtype == GOFANN_DTYPE_U8) {
            for (int i = lane; i < len; i += kWarp) {
                const uint32_t s = __float_as_uint(dist[i]);
                dist[i] = static_cast<float>(l2_u8_thread(basep + static_cast<size_t>(s) * row_bytes,
                                                          reinterpret_cast<const uint4*>(q), n16, stream));
            }
        } else {
            for (int i0 = 0; i0 < len; i0 += 4) {
                const void* rows[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    rows[u] = i0 + u < len ? basep + static_cast<size_t>(__float_as_uint(dist[i0 + u])) * row_bytes
                                           : nullptr;
                float o[4];
                l2_float_warp<kDtype, 4>(rows, q, static_cast<int>(a.dim), lane, stream, o);
                __syncwarp();
                if (lane == 0) {
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (i0 + u < len) dist[i0 + u] = o[u];
                }
            }
        }
        __syncwarp();

        // admissions in edge order (backend_full_gpu.cu:1976-1994)
        const bool full = hs > 2 && hs >= QS + 1;
        const float maxv = full ? h.key[2] : 0.0f;
        uint32_t rej[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int i = hh * kWarp + lane;
            rej[hh] = __ballot_sync(kFull, i < len && full && maxv < dist[i]);
        }
        uint32_t adm[2] = {0u, 0u};
        int n_adm = 0;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int n_here = len - hh * kWarp;
            unsigned todo = n_here <= 0 ? 0u : ~rej[hh] & (n_here >= kWarp ? kFull : (1u << n_here) - 1u);
            while (todo) {
                const int i = hh * kWarp + __ffs(todo) - 1;
                todo &= todo - 1;
                const float key = dist[i];
                if (hs > 2 && hs >= QS + 1 && h.key[2] < key) continue;
                smmh_insert_warp(h, hs, key, list[i], key, lane);
                ++hs;
                adm[hh] |= 1u << (i & 31);
                ++n_adm;
                if (hs >= QS + 2) {
                    smmh_pop_max_warp(h, hs, lane);
                    --hs;
                }
            }
        }
        n_adm_total += static_cast<uint32_t>(n_adm);
        // visited-table inserts of the admitted rows (absent until now: they
        // passed this step's test, and nothing reads the table before the next
        // step); concurrent plain stores into the slots their tests saw, or
        // one by one when the table could fill or an id repeats
        {
            bool serial = hash_count + n_adm > kHashCap;
            int slot[2] = {-1, -1};
            if (!serial) {
                bool repeat = false;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int i = hh * kWarp + lane;
                    if ((adm[hh] >> lane) & 1u) {
                        const uint32_t b = cbucket[i];
                        int rank = 0;
#pragma unroll
                        for (int h2 = 0; h2 < 2; ++h2) {
                            uint32_t before = adm[h2];
                            if (h2 > hh) before = 0u;
                            else if (h2 == hh) before &= (1u << lane) - 1u;
                            while (before) {
                                const int j = h2 * kWarp + __ffs(before) - 1;
                                before &= before - 1;
                                if (cbucket[j] == b) {
                                    ++rank;
                                    repeat |= list[j] == list[i];
                                }
                            }
                        }
                        const int sl = nth_set_bit(cfree[i], rank);
                        slot[hh] = sl >= 0 ? sl : -2;
                    }
                }
                serial = __any_sync(kFull, repeat);
            }
            if (serial) {
                int added = 0;
                if (lane == 0)
                    for (int i = 0; i < len; ++i)
                        if (((i < kWarp ? adm[0] : adm[1]) >> (i & 31)) & 1u) added += hash_add(hash, list[i]) ? 1 : 0;
                hash_count += __shfl_sync(kFull, added, 0);
            } else {
                hash_count += n_adm;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh)
                    if (slot[hh] >= 0) hash[cbucket[hh * kWarp + lane] * kBucketSlots + slot[hh]] = list[hh * kWarp + lane];
                __syncwarp();
#pragma unroll
                for (int hh = 0; hh < 2; ++hh)
                    if (slot[hh] == -2) hash_add_concurrent(hash, list[hh * kWarp + lane]);
            }
        }
        __syncwarp();

        // next node and the stop rule (backend_full_gpu.cu:1997-2031)
        const int bi = pickup(h, hs, lane);
        if (bi < 0) break;
        const float next_key = h.key[bi];
        const uint32_t next_val = h.val[bi];
        __syncwarp();
        if (lane == 0) h.val[bi] |= kPoolUsed;
        const uint32_t next_local = next_val & ~kPoolUsed;
        {
            const uint32_t* src = a.graph.adjacency + static_cast<size_t>(off + next_local) * a.graph.degree;
            for (int hh = 0; hh < 2; ++hh) {
                const uint32_t i = hh * kWarp + lane;
                nb[hh] = i < deg ? ldg_u32(src + i, stream) : kU32Max;
            }
        }
        if (!first_step) {
            const uint32_t next_sample = a.graph.row_to_sample[off + next_local];
            if (p.early_stop_mode == GOFANN_EARLY_STOP_ADAPTIVE && improved) {
                fh = 0;
            } else if (best.size == K &&
                       !better(next_key, next_sample, __shfl_sync(kFull, best.d, K - 1),
                               __shfl_sync(kFull, best.id, K - 1))) {
                ++fh;
                if (early_stop_reached(p.early_stop_mode, fh, p.finish_limit, QS, expanded, passed, K)) break;
            } else {
                fh = 0;
            }
        }
        now_key = next_key;
        now_val = next_val;
        first_step = false;
        // the next step's visited-table lines and row -> sample entries
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            if (nb[hh] != kU32Max && nb[hh] < gsize) {
                prefetch_l1(hash + home_bucket(nb[hh]) * kBucketSlots);
                prefetch_l2(a.graph.row_to_sample + off + nb[hh]);
            }
        }
        __syncwarp();
    }

    // results: sample ids ascending by (distance, id), UINT32_MAX / FLT_MAX fill
    uint32_t* oid = a.out.ids + static_cast<size_t>(route) * K;
    float* od = a.out.dists + static_cast<size_t>(route) * K;
    if (lane < K) {
        oid[lane] = lane < best.size ? best.id : kU32Max;
        od[lane] = lane < best.size ? best.d : FLT_MAX;
    }
    if (a.out.trace)
        for (uint32_t i = static_cast<uint32_t>(expanded) + lane; i < a.out.trace_width; i += kWarp)
            a.out.trace[static_cast<size_t>(route) * a.out.trace_width + i] = kU32Max;
    if (lane == 0) {
        if (a.out.steps) a.out.steps[route] = steps;
        if (a.out.counters) {
            uint32_t* c = a.out.counters + static_cast<size_t>(route) * 4;
            c[0] = static_cast<uint32_t>(expanded);
            c[1] = n_dist;
            c[2] = static_cast<uint32_t>(passed);
            c[3] = n_adm_total;
        }
    }
    __syncwarp();
}

template <int kDtype>
__global__ void __launch_bounds__(kBlockWarps * 32, 6) exact_search_kernel(ExactArgs a)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    unsigned char* wbase = smem_raw + static_cast<size_t>(warp) * a.warp_smem;
    const uint32_t gwarp = blockIdx.x * (blockDim.x >> 5) + warp;
    uint32_t* hash = a.hash + static_cast<size_t>(gwarp) * kHashCap;
    const uint64_t stream = l2_stream_policy();
    for (;;) {
        uint32_t route = 0;
        if (lane == 0) route = atomicAdd(a.route_counter, 1u);
        route = __shfl_sync(kFull, route, 0);
        if (route >= a.routes.n_routes) break;
        run_route<kDtype>(a, wbase, hash, route, lane, stream);
    }
}

}  // namespace exact
}  // namespace gofann

using namespace gofann;

extern "C" {

size_t gofann_exact_search_scratch_bytes(uint32_t n_routes)
{
    const uint32_t sms = static_cast<uint32_t>(sm_count() > 0 ? sm_count() : 148);
    uint64_t warps = static_cast<uint64_t>(n_routes) + exact::kBlockWarps - 1;
    const uint64_t cap = static_cast<uint64_t>(sms) * 64;
    if (warps > cap) warps = cap;
    if (warps == 0) warps = exact::kBlockWarps;
    return exact::kCounterBytes + warps * kHashCap * sizeof(uint32_t);
}

int gofann_exact_search(const gofann_graph* graph, const uint32_t* label_size, const gofann_attrs* attrs,
                        const void* base, int dtype, uint32_t dim, const void* queries, const gofann_routes* routes,
                        const gofann_search_params* params, const gofann_search_out* out, void* scratch,
                        size_t scratch_bytes, void* stream)
{
    if (!graph || !attrs || !base || !queries || !routes || !params || !out || !scratch)
        return fail(GOFANN_ERR_INVALID, "exact_search: null argument");
    const gofann_search_params& p = *params;
    if (p.queue_size < 2 || p.queue_size > GOFANN_MAX_QUEUE)
        return fail(GOFANN_ERR_INVALID, "exact_search: queue_size %d outside 2..%d", p.queue_size, GOFANN_MAX_QUEUE);
    if (p.result_width < 1 || p.result_width > GOFANN_MAX_TOPK)
        return fail(GOFANN_ERR_INVALID, "exact_search: result_width (topk) %d outside 1..%d", p.result_width,
                    GOFANN_MAX_TOPK);
    if (p.early_stop_mode < 0 || p.early_stop_mode > 2)
        return fail(GOFANN_ERR_INVALID, "exact_search: unknown early_stop_mode %d", p.early_stop_mode);
    if (p.max_steps < 0) return fail(GOFANN_ERR_INVALID, "exact_search: max_steps %d is negative", p.max_steps);
    if (!graph->adjacency || !graph->row_to_sample || !graph->label_offset || graph->degree == 0)
        return fail(GOFANN_ERR_INVALID, "exact_search: graph arrays missing");
    if (!routes->query_row || !routes->group_id || !routes->start_local || !out->ids || !out->dists)
        return fail(GOFANN_ERR_INVALID, "exact_search: route or output arrays missing");
    if ((routes->qlabel_indptr || routes->range_modes) && (!attrs->label_indptr || !attrs->label_indices))
        return fail(GOFANN_ERR_INVALID, "exact_search: residual labels need the sample label CSR");
    if (dtype != GOFANN_DTYPE_U8 && dtype != GOFANN_DTYPE_F32 && dtype != GOFANN_DTYPE_F16)
        return fail(GOFANN_ERR_INVALID, "exact_search: unknown dtype %d", dtype);
    const uint32_t elem = dtype == GOFANN_DTYPE_U8 ? 1u : (dtype == GOFANN_DTYPE_F16 ? 2u : 4u);
    if (dim == 0 || (dim * elem) % 16 != 0 || dim * elem > 16384)
        return fail(GOFANN_ERR_UNSUPPORTED, "exact_search: rows of %u x %u bytes (need a multiple of 16, <= 16 KB)",
                    dim, elem);
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (reinterpret_cast<uintptr_t>(queries) & 15) != 0)
        return fail(GOFANN_ERR_INVALID, "exact_search: base and queries must be 16-byte aligned");
    if (routes->n_routes == 0) return GOFANN_OK;

    exact::ExactArgs a{};
    a.graph = *graph;
    a.label_size = label_size;
    a.attrs = make_attr_view(attrs);
    a.routes = *routes;
    a.p = p;
    a.out = *out;
    a.base = base;
    a.queries = queries;
    a.dim = dim;
    a.status = out->status;
    const exact::Layout L = exact::layout(p.queue_size, dim, elem);
    a.warp_smem = L.total;
    const int wpb = exact::kBlockWarps;
    const size_t smem = static_cast<size_t>(L.total) * wpb;
    if (smem > 227 * 1024) return fail(GOFANN_ERR_UNSUPPORTED, "exact_search: %zu bytes of shared memory", smem);
    void (*kern)(exact::ExactArgs) = dtype == GOFANN_DTYPE_U8    ? exact::exact_search_kernel<GOFANN_DTYPE_U8>
                                     : dtype == GOFANN_DTYPE_F16 ? exact::exact_search_kernel<GOFANN_DTYPE_F16>
                                                                 : exact::exact_search_kernel<GOFANN_DTYPE_F32>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e, "exact_search: shared memory attribute");
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, wpb * 32, smem);
    if (e != cudaSuccess) return cuda_status(e, "exact_search: occupancy query");
    if (per_sm <= 0) return fail(GOFANN_ERR_UNSUPPORTED, "exact_search: kernel does not fit on an SM");
    const uint32_t need = (routes->n_routes + wpb - 1) / wpb;
    uint32_t blocks = static_cast<uint32_t>(per_sm) * static_cast<uint32_t>(sm_count() > 0 ? sm_count() : 148);
    if (p.resident_warps > 0) {
        const uint32_t capb = static_cast<uint32_t>((p.resident_warps + wpb - 1) / wpb);
        if (capb < blocks) blocks = capb;
    }
    if (need < blocks) blocks = need;
    const size_t need_bytes = exact::kCounterBytes + static_cast<size_t>(blocks) * wpb * kHashCap * sizeof(uint32_t);
    if (scratch_bytes < need_bytes)
        return fail(GOFANN_ERR_CAPACITY, "exact_search: scratch of %zu bytes, %zu needed", scratch_bytes, need_bytes);
    a.route_counter = static_cast<uint32_t*>(scratch);
    a.hash = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(scratch) + exact::kCounterBytes);
    cudaStream_t s = as_stream(stream);
    e = cudaMemsetAsync(scratch, 0, sizeof(uint32_t), s);
    if (e != cudaSuccess) return cuda_status(e, "exact_search: counter reset");
    kern<<<blocks, wpb * 32, smem, s>>>(a);
    GOFANN_CHECK_LAUNCH("exact_search_kernel");
    return GOFANN_OK;
}

}  // extern "C"
