// common.cuh — shared device helpers of the B200 filtered-ANN search path.
//
// Host side: thread-local error string + status helpers used by every C-ABI
// entry point.  Device side: the data-structure algorithms whose exact
// behaviour decides which ids a traversal returns (visited hash, symmetric
// min-max frontier, binary result heaps, (dist,id) ordering), the DNF
// predicate, and the warp-order replays of the reference's float reductions.
#pragma once

#include <cfloat>
#include <cstdint>
#include <cstdio>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/gofann.h"

namespace gofann {

// ----------------------------------------------------------------- host
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
int cuda_status(cudaError_t err, const char* what);
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
int sm_count();
size_t l2_bytes();  // L2 size of the current device (0 on error)

#define GOFANN_CHECK_LAUNCH(what)                                      \
    do {                                                               \
        cudaError_t _e = cudaGetLastError();                           \
        if (_e != cudaSuccess) return ::gofann::cuda_status(_e, what); \
    } while (0)

constexpr uint32_t kU32Max = 0xffffffffu;
constexpr uint32_t kPoolUsed = 0x80000000u;
constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kHashCap = GOFANN_HASH_CAPACITY;

// ---------------------------------------------------- L2 residency classes
// A traversal re-reads its route's tables (the 48 KB PQ lookup row at
// config-2 shape) for every candidate of every step, but reads graph rows,
// code rows and the row->sample map about once per route.  With thousands of
// routes in flight the tables alone approach the L2 size, so plain LRU lets
// the streaming reads evict them and the table gathers fall through to HBM as
// 32-byte sectors.  Table loads therefore carry an L2 evict_last policy and
// streaming loads an evict_first policy (PTX createpolicy + .L2::cache_hint).
// Policies change only caching, never values.
__device__ __forceinline__ uint64_t l2_keep_policy()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_stream_policy()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Read-only (non-coherent) global loads with a cache policy; the data must
// not be written while the kernel runs.
__device__ __forceinline__ float ldg_f32(const float* p, uint64_t pol)
{
    float v;
    asm volatile("ld.global.nc.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ float4 ldg_f32x4(const float4* p, uint64_t pol)
{
    float4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ uint32_t ldg_u32(const uint32_t* p, uint64_t pol)
{
    uint32_t v;
    asm volatile("ld.global.nc.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ uint4 ldg_u32x4(const uint4* p, uint64_t pol)
{
    uint4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}

// Non-blocking fetch of the line holding p into L1 or L2 (PTX prefetch): the
// traversal issues them one step ahead for the rows the next step reads, so
// that those reads do not wait on HBM or L2.
__device__ __forceinline__ void prefetch_l1(const void* p)
{
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}
__device__ __forceinline__ void prefetch_l2(const void* p)
{
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// --------------------------------------------------- float order helpers
// Lane-0 value of `v += __shfl_xor_sync(v, off)` for off = 16..1, replayed
// inside one thread from the 32 lane partials (backend_pq.cu:4716-4721).
// Float addition is commutative, so lane i's step v[i] + v[i^off] equals
// v[i] + v[i+off] for the lanes (i < off) that lane 0 depends on.
__device__ __forceinline__ float butterfly_sum32(float (&v)[32])
{
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
        for (int i = 0; i < off; ++i) v[i] = __fadd_rn(v[i], v[i + off]);
    }
    return v[0];
}

// ------------------------------------------------------------ visited hash
// native_visited_hash.cuh:11-61: multiplicative mix modulo 4096, UINT32_MAX
// = empty, a full table silently drops the insert.
__device__ __forceinline__ uint32_t hash_code(uint32_t v)
{
    const uint64_t mixed = static_cast<uint64_t>(v) ^
                           (static_cast<uint64_t>(v >> 16) * 0x4bcb391f924ed183ULL) ^
                           0xa0ab69ccd854fc0aULL;
    return static_cast<uint32_t>(mixed % kHashCap);
}
// The traversal's tables use a bucketed layout of the same 4,096 slots.  The
// reference's table answers one question -- was this row inserted -- and
// drops an insert exactly when all 4,096 slots are taken; any exact set of
// 4,096 slots with that rule answers identically.  Here the slots form 512
// buckets of 8 (one 32-byte sector); a value's home bucket is
// hash_code(v) / 8, and a value lives in the first bucket of its probe
// sequence (home, home + 1, ... mod 512) that had a free slot when it was
// inserted.  Nothing is ever removed, so a bucket holding a free slot ends
// every probe sequence that reaches it: a test reads one sector, and the
// free-slot mask it sees tells where the value would go.
constexpr int kBucketSlots = 8;
constexpr int kBuckets = kHashCap / kBucketSlots;

__device__ __forceinline__ uint32_t home_bucket(uint32_t v) { return hash_code(v) / kBucketSlots; }

struct BucketProbe {
    uint32_t bucket;     // bucket holding v, or the first with a free slot (kU32Max: table full)
    uint32_t free_mask;  // free slots of that bucket (bit j = slot j)
    bool found;
};
__device__ __forceinline__ BucketProbe bucket_probe(const uint32_t* t, uint32_t v)
{
    uint32_t b = home_bucket(v);
    for (int n = 0; n < kBuckets; ++n) {
        const uint4* q = reinterpret_cast<const uint4*>(t + b * kBucketSlots);
        const uint4 x = q[0], y = q[1];
        const uint32_t w[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
        uint32_t fm = 0;
        bool hit = false;
#pragma unroll
        for (int j = 0; j < kBucketSlots; ++j) {
            hit = hit || w[j] == v;
            fm |= (w[j] == kU32Max ? 1u : 0u) << j;
        }
        if (hit) return {b, fm, true};
        if (fm) return {b, fm, false};
        b = (b + 1) & (kBuckets - 1);
    }
    return {kU32Max, 0u, false};
}
__device__ __forceinline__ bool hash_test(const uint32_t* t, uint32_t v) { return bucket_probe(t, v).found; }
// Returns true when v was inserted (false: already present, or table full).
__device__ __forceinline__ bool hash_add(uint32_t* t, uint32_t v)
{
    const BucketProbe pr = bucket_probe(t, v);
    if (pr.found || pr.bucket == kU32Max) return false;
    t[pr.bucket * kBucketSlots + __ffs(pr.free_mask) - 1] = v;
    return true;
}
// Concurrent insertion of distinct absent values by several lanes, with
// atomics: the slot a value lands in can differ from the one-at-a-time
// order, but membership -- the only thing a test reads -- is the same as long
// as the table cannot fill, which the caller guarantees.
__device__ __forceinline__ void hash_add_concurrent(uint32_t* t, uint32_t v)
{
    uint32_t b = home_bucket(v);
    for (int n = 0; n < kBuckets; ++n) {
        for (int j = 0; j < kBucketSlots; ++j) {
            const uint32_t x = atomicCAS(t + b * kBucketSlots + j, kU32Max, v);
            if (x == kU32Max || x == v) return;
        }
        b = (b + 1) & (kBuckets - 1);
    }
}
// k-th set bit (0-based) of m, or -1.
__device__ __forceinline__ int nth_set_bit(uint32_t m, int k)
{
    for (int r = 0; r < k; ++r) m &= m - 1;
    return m ? __ffs(m) - 1 : -1;
}

// ---------------------------------------------------------------- frontier
// Frontier entry: priority, local row | used bit, unbiased score
// (gpu_predicate::BiasedPair, gpu_predicate_index.cuh:137-144).
struct FPair {
    float first;
    uint32_t second;
    float base;
};

// The reference's frontier is a symmetric min-max heap (include/smmh2.h:
// 8-148: index 0 unused, 1 = min, 2 = max, entries compared by `first`).
// Here it is stored as three arrays (key = `first`, val = payload, base =
// unbiased score) and operated on by a whole warp.  Every lane runs the
// same, warp-uniform sequence of the reference's decisions on broadcast
// shared-memory reads; lane 0 writes.  Only the fetching is parallel:
//   * insert: the new element climbs the chain of ancestor pairs fixed by
//     its leaf position; at each pair the reference compares it strictly with
//     the left (min) element, then the right (max) one, and once it moves up
//     one side it can never satisfy the other side's test again (the heap
//     order), so lane j reads the pair j levels up, a ballot over "strictly
//     below the left" (or "strictly above the right") gives the number of
//     levels climbed -- the leading passed levels, exactly where the
//     reference stops -- and the displaced elements move down one level
//     together;
//   * pop_max: the sift-down stays sequential (each level depends on the
//     previous one); the moving element lives in registers and a level's
//     sibling and child entries are read together.
struct Smmh {
    float* key;
    uint32_t* val;
    float* base;
};

// Inserts (ek, ev, eb) into a heap whose next free index is `size` (entries
// + 1); the caller increments its size.
__device__ __forceinline__ void smmh_insert_warp(const Smmh& h, int size, float ek, uint32_t ev, float eb, int lane)
{
    int y = size;
    if ((y & 1) == 0) {  // adjust_sibling at the leaf: a right child below its left sibling swaps
        const float sk = h.key[y - 1];
        if (ek < sk) {
            if (lane == 0) {
                h.key[y] = sk;
                h.val[y] = h.val[y - 1];
                h.base[y] = h.base[y - 1];
            }
            y -= 1;
        }
    }
    if (y > 2) {
        const int p0 = (y - 1) >> 1;              // pair of y; pair P's elements are 2P+1, 2P+2
        const int levels = 31 - __clz(p0 + 1);    // ancestor pairs above it
        bool up_min = false, up_max = false;
        if (lane >= 1 && lane <= levels) {
            const int P = ((p0 + 1) >> lane) - 1;
            up_min = h.key[2 * P + 1] > ek;
            up_max = h.key[2 * P + 2] < ek;
        }
        const unsigned bmin = __ballot_sync(kFull, up_min) >> 1;  // bit j-1: pair j levels up
        const unsigned bmax = __ballot_sync(kFull, up_max) >> 1;
        int side = 0;
        unsigned passed = 0;
        if (bmin & 1u) { side = 1; passed = bmin; }
        else if (bmax & 1u) { side = 2; passed = bmax; }
        if (side != 0) {
            const int climb = __ffs(~passed) - 1;
            const bool mover = lane >= 1 && lane <= climb;
            float mk = 0.0f, mb = 0.0f;
            uint32_t mv = 0;
            int dst = 0;
            if (mover) {
                const int src = 2 * (((p0 + 1) >> lane) - 1) + side;
                mk = h.key[src];
                mv = h.val[src];
                mb = h.base[src];
                dst = lane == 1 ? y : 2 * (((p0 + 1) >> (lane - 1)) - 1) + side;
            }
            __syncwarp();
            if (mover) {
                h.key[dst] = mk;
                h.val[dst] = mv;
                h.base[dst] = mb;
            }
            y = 2 * (((p0 + 1) >> climb) - 1) + side;
        }
    }
    __syncwarp();
    if (lane == 0) {
        h.key[y] = ek;
        h.val[y] = ev;
        h.base[y] = eb;
    }
    __syncwarp();
}

// Removes the maximum (index 2) of a heap of `size` - 1 entries; the caller
// decrements its size.  Needs at least 3 entries (`size` >= 4), which the
// traversal guarantees (it pops only above queue_size + 1 >= 3 entries).
__device__ __forceinline__ void smmh_pop_max_warp(const Smmh& h, int size, int lane)
{
    --size;
    float ck = h.key[size];  // h[2] = h[--size]
    uint32_t cv = h.val[size];
    float cb = h.base[size];
    int y = 2;  // stays a right (even) index
    for (;;) {
        const int s = y - 1, cl = 2 * y, cr = 2 * y + 2;
        const float sk = h.key[s];
        const uint32_t sv = h.val[s];
        const float sb = h.base[s];
        float lk = 0.0f, lb = 0.0f, rk = 0.0f, rb = 0.0f;
        uint32_t lv = 0, rv = 0;
        if (cl < size) { lk = h.key[cl]; lv = h.val[cl]; lb = h.base[cl]; }
        if (cr < size) { rk = h.key[cr]; rv = h.val[cr]; rb = h.base[cr]; }
        // adjust_sibling (the reference's pop_max ignores the index it returns)
        if (ck < sk) {
            if (lane == 0) {
                h.key[s] = ck;
                h.val[s] = cv;
                h.base[s] = cb;
            }
            ck = sk; cv = sv; cb = sb;
        }
        // adjust_grandchild: the larger right child of the two child pairs
        if (cl >= size) break;
        bool right = cr < size && rk > lk;
        const float chk = right ? rk : lk;
        if (!(chk > ck)) break;
        if (lane == 0) {
            h.key[y] = chk;
            h.val[y] = right ? rv : lv;
            h.base[y] = right ? rb : lb;
        }
        y = right ? cr : cl;
    }
    if (lane == 0) {
        h.key[y] = ck;
        h.val[y] = cv;
        h.base[y] = cb;
    }
    __syncwarp();
}

// -------------------------------------------------------- binary max heaps
// include/bin_heap.h:6-66 over entries with a float key `first`.
template <class T>
__device__ __forceinline__ void bheap_push(T* b, int n)
{
    int now = n - 1;
    int parent = (now - 1) / 2;
    while (now > 0 && b[parent].first < b[now].first) {
        T t = b[now]; b[now] = b[parent]; b[parent] = t;
        now = parent;
        parent = (now - 1) / 2;
    }
}
template <class T>
__device__ __forceinline__ T bheap_pop(T* b, int n)
{
    T ret = b[0];
    const int len = n - 1;
    if (len <= 0) return ret;
    b[0] = b[n - 1];
    int now = 0;
    while (now * 2 + 1 < len) {
        const int l = now * 2 + 1, r = now * 2 + 2;
        int nx = l;
        if (r < len && b[l].first < b[r].first) nx = r;
        if (!(b[now].first < b[nx].first)) break;
        T t = b[now]; b[now] = b[nx]; b[nx] = t;
        now = nx;
    }
    return ret;
}
struct RPair { float first; uint32_t second; };             // ResultPair
struct SPair { float first; uint32_t pad; uint64_t second; }; // stop top-k entry

// (dist, id) lexicographic order of posting_shortlist_heap.cuh:14-20.
__device__ __forceinline__ bool pair_less(float ld, uint32_t li, float rd, uint32_t ri)
{
    return ld < rd || (ld == rd && li < ri);
}

// ---------------------------------------------------------------- filters
struct AttrView {
    const uint64_t* indptr;
    const uint32_t* indices;
    const float* ranges;
    uint32_t n_samples;
    uint32_t range_count;
    const uint64_t* str_offsets;
    const uint8_t* str_bytes;
    const int64_t* ints;
    uint32_t int_count;
};
// The device view of a gofann_attrs descriptor (zeros for NULL).
inline AttrView make_attr_view(const gofann_attrs* a)
{
    AttrView v{};
    if (a) {
        v.indptr = a->label_indptr;
        v.indices = a->label_indices;
        v.ranges = a->range_values;
        v.n_samples = a->n_samples;
        v.range_count = a->range_count;
        v.str_offsets = a->string_offsets;
        v.str_bytes = a->string_bytes;
        v.ints = a->int_values;
        v.int_count = a->int_count;
    }
    return v;
}

// Is `label` in the sorted label row indices[begin, end)?
__device__ __forceinline__ bool row_contains(const uint32_t* indices, uint64_t begin, uint64_t end, uint32_t label)
{
    uint64_t lo = begin, hi = end;
    while (lo < hi) {
        const uint64_t mid = lo + ((hi - lo) >> 1);
        const uint32_t v = indices[mid];
        if (v < label) lo = mid + 1; else hi = mid;
    }
    return lo < end && indices[lo] == label;
}
__device__ __forceinline__ bool csr_contains(const AttrView& a, uint32_t sample, uint32_t label)
{
    return row_contains(a.indices, a.indptr[sample], a.indptr[sample + 1], label);
}
__device__ __forceinline__ bool range_match(uint32_t mode, float lo, float hi, float v)
{
    switch (mode) {
    case 0: return true;
    case 1: return v > lo;
    case 2: return v < hi;
    case 3: return v >= lo && v < hi;
    default: return false;
    }
}
__device__ __forceinline__ bool pred_enabled(const gofann_routes& r, uint32_t route)
{
    if (!r.pred_offsets) return false;
    return r.pred_enabled ? r.pred_enabled[route] != 0 : true;
}
// Levenshtein distance between a pattern of m <= 32 bytes (its match table
// peq: bit i of peq[c] = pattern[i] == c) and text[0, n), by the
// bit-parallel algorithm of Myers (J. ACM 46(3), 1999) in the global form of
// Hyyro (2001): column j of the DP matrix is kept as vertical +1 / -1 delta
// bit vectors, the top row D[0][j] = j contributes a horizontal +1 carried
// into bit 0, and the last row's value is tracked in `score`.  Text bytes
// of 128 and above match no pattern byte.
__device__ __forceinline__ uint32_t myers_edit_distance(const uint32_t* __restrict__ peq, uint32_t m,
                                                        const uint8_t* __restrict__ text, uint32_t n)
{
    if (m == 0) return n;
    const uint32_t last = 1u << (m - 1);
    uint32_t pv = m == 32 ? 0xffffffffu : (1u << m) - 1u, mv = 0u, score = m;
    for (uint32_t j = 0; j < n; ++j) {
        const uint8_t c = text[j];
        const uint32_t eq = c < 128 ? __ldg(peq + c) : 0u;
        const uint32_t xv = eq | mv;
        const uint32_t xh = (((eq & pv) + pv) ^ pv) | eq;
        uint32_t ph = mv | ~(xh | pv);
        uint32_t mh = pv & xh;
        if (ph & last) ++score;
        else if (mh & last) --score;
        ph = (ph << 1) | 1u;
        mh <<= 1;
        pv = mh | ~(xv | ph);
        mv = ph & xv;
    }
    return score;
}

// String and integer atoms of clause `ci` for `sample` (all must hold).
// Not inlined, and given plain pointers: the traversal's step loop calls it
// only for routes whose clauses carry such atoms, and neither its code nor
// a copy of the descriptors enters the hot loop.
static __device__ __noinline__ bool ext_atoms_match(const gofann_clause_ext* __restrict__ ext,
                                                    const gofann_int_atom* __restrict__ int_atoms,
                                                    const gofann_string_atom* __restrict__ str_atoms,
                                                    const uint8_t* __restrict__ str_query,
                                                    const uint32_t* __restrict__ peq_rows,
                                                    const int64_t* __restrict__ ints, uint32_t int_count,
                                                    const uint64_t* __restrict__ str_offsets,
                                                    const uint8_t* __restrict__ str_bytes, uint32_t ci,
                                                    uint32_t sample)
{
    const gofann_clause_ext x = ext[ci];
    for (uint32_t j = x.int_begin; j < x.int_end; ++j) {
        const gofann_int_atom at = int_atoms[j];
        if (at.mode == 0) continue;
        if (ints == nullptr || at.dimension >= int_count) return false;
        const int64_t v = ints[static_cast<uint64_t>(sample) * int_count + at.dimension];
        const bool ok = at.mode == 1 ? v > at.lower : at.mode == 2 ? v < at.upper
                                                     : at.mode == 3 ? (v >= at.lower && v < at.upper) : false;
        if (!ok) return false;
    }
    if (x.string_begin == x.string_end) return true;
    if (str_offsets == nullptr) return false;
    const uint64_t sb = str_offsets[sample], se = str_offsets[sample + 1];
    const uint8_t* text = str_bytes + sb;
    const uint32_t n = static_cast<uint32_t>(se - sb);
    for (uint32_t j = x.string_begin; j < x.string_end; ++j) {
        const gofann_string_atom at = str_atoms[j];
        const uint8_t* q = str_query + at.offset;
        if (at.kind == GOFANN_STRING_EXACT) {
            if (n != at.length) return false;
            for (uint32_t i = 0; i < n; ++i)
                if (text[i] != q[i]) return false;
        } else {
            const uint32_t gap = n > at.length ? n - at.length : at.length - n;
            if (gap > at.max_edits || at.length > GOFANN_FUZZY_MAX_LENGTH) return false;
            if (myers_edit_distance(peq_rows + static_cast<size_t>(j) * 128, at.length, text, n) > at.max_edits)
                return false;
        }
    }
    return true;
}
__device__ __forceinline__ bool ext_atoms_match(const gofann_routes& r, const AttrView& a, uint32_t ci,
                                                uint32_t sample)
{
    return ext_atoms_match(r.pred_ext, r.pred_ints, r.pred_strings, r.pred_string_bytes, r.pred_string_peq, a.ints,
                           a.int_count, a.str_offsets, a.str_bytes, ci, sample);
}

// gpu_predicate::matches with clauses (gpu_predicate_index.cuh:109-136),
// given the sample's sorted label row labels[lbegin, lend) (the CSR's
// indices, or a copy of the row), then the clause's string and integer
// atoms when the routes carry them (kExt: traversal variants compiled with
// kExt = false serve routes without such atoms, with no trace of the check
// in their code).
template <bool kExt = true>
__device__ __forceinline__ bool pred_matches_row(const gofann_routes& r, const AttrView& a, uint32_t route,
                                                 uint32_t sample, const uint32_t* labels, uint64_t lbegin,
                                                 uint64_t lend)
{
    if (sample >= a.n_samples) return false;
    const uint32_t e = r.pred_offsets[route + 1];
    for (uint32_t i = r.pred_offsets[route]; i < e; ++i) {
        const gofann_clause c = r.clauses[i];
        bool pass = true;
        for (uint32_t j = c.label_begin; pass && j < c.label_end; ++j)
            pass = row_contains(labels, lbegin, lend, r.pred_handles[j]);
        for (uint32_t j = c.range_begin; pass && j < c.range_end; ++j) {
            const gofann_range_atom at = r.pred_ranges[j];
            pass = a.ranges != nullptr && at.dimension < a.range_count &&
                   range_match(at.mode, at.lower, at.upper,
                               a.ranges[static_cast<uint64_t>(sample) * a.range_count + at.dimension]);
        }
        if (kExt && pass && r.pred_ext) pass = ext_atoms_match(r, a, i, sample);
        if (pass) return true;
    }
    return false;
}
// gpu_predicate::matches with clauses (gpu_predicate_index.cuh:109-136),
// plus the clauses' string and integer atoms.
template <bool kExt = true>
__device__ __forceinline__ bool pred_matches(const gofann_routes& r, const AttrView& a,
                                             uint32_t route, uint32_t sample)
{
    if (sample >= a.n_samples) return false;
    const uint32_t e = r.pred_offsets[route + 1];
    for (uint32_t i = r.pred_offsets[route]; i < e; ++i) {
        const gofann_clause c = r.clauses[i];
        bool pass = true;
        for (uint32_t j = c.label_begin; pass && j < c.label_end; ++j)
            pass = csr_contains(a, sample, r.pred_handles[j]);
        for (uint32_t j = c.range_begin; pass && j < c.range_end; ++j) {
            const gofann_range_atom at = r.pred_ranges[j];
            pass = a.ranges != nullptr && at.dimension < a.range_count &&
                   range_match(at.mode, at.lower, at.upper,
                               a.ranges[static_cast<uint64_t>(sample) * a.range_count + at.dimension]);
        }
        if (kExt && pass && r.pred_ext) pass = ext_atoms_match(r, a, i, sample);
        if (pass) return true;
    }
    return false;
}
// resident_pq_labels_match (backend_pq.cu:3934-3965): every query label but
// the route's primary one must be in the sample's row.
__device__ __forceinline__ bool labels_match(const gofann_routes& r, const AttrView& a,
                                             uint32_t route, uint32_t sample)
{
    if (!r.qlabel_indptr) return true;
    const uint32_t primary = r.primary_label ? r.primary_label[route] : kU32Max;
    const uint64_t e = r.qlabel_indptr[route + 1];
    for (uint64_t p = r.qlabel_indptr[route]; p < e; ++p) {
        const uint32_t l = r.qlabel_indices[p];
        if (l == primary) continue;
        if (!csr_contains(a, sample, l)) return false;
    }
    return true;
}
// gpu_predicate::priority (gpu_predicate_index.cuh:161-166).
__device__ __forceinline__ float pred_priority(float base, float penalty, bool pass)
{
    if (pass || penalty == 0.0f || !isfinite(base) || base == FLT_MAX) return base;
    if (base > FLT_MAX - penalty) return FLT_MAX;
    return __fadd_rn(base, penalty);
}

// ------------------------------------------------------------ warp top-k
// Smallest (dist, id) pairs with unique ids among `n` entries, selected by
// `k` rounds of warp argmin.  An entry whose id was already taken is
// skipped: an id's first selection carries its minimum distance, so the
// result equals "dedup by id keeping the minimum distance, sort by
// (dist, id), truncate to k" (rabitq_lowfreq_merge.h:773-813).  `get(i, d,
// id)` loads entry i from any memory.  Lane 0 writes the k outputs.
template <int kMaxK, class Get>
__device__ __forceinline__ void warp_select_topk(int n, int k, Get get, uint32_t* out_ids, float* out_d,
                                                 int lane)
{
    uint32_t sel[kMaxK];
#pragma unroll
    for (int r = 0; r < kMaxK; ++r) sel[r] = kU32Max;
    for (int r = 0; r < k; ++r) {
        float bd = FLT_MAX;
        uint32_t bi = kU32Max;
        int found = 0;
        for (int i = lane; i < n; i += kWarp) {
            float x;
            uint32_t y;
            get(i, x, y);
            if (y == kU32Max) continue;
            bool taken = false;
#pragma unroll
            for (int t = 0; t < kMaxK; ++t) taken |= (t < r) && sel[t] == y;
            if (taken) continue;
            if (!found || pair_less(x, y, bd, bi)) { bd = x; bi = y; found = 1; }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float od = __shfl_xor_sync(kFull, bd, off);
            const uint32_t oi = __shfl_xor_sync(kFull, bi, off);
            const int of = __shfl_xor_sync(kFull, found, off);
            if (of && (!found || pair_less(od, oi, bd, bi))) { bd = od; bi = oi; found = 1; }
        }
        if (lane == 0) {
            out_ids[r] = found ? bi : kU32Max;
            out_d[r] = found ? bd : FLT_MAX;
        }
#pragma unroll
        for (int t = 0; t < kMaxK; ++t)
            if (t == r) sel[t] = found ? bi : kU32Max;
    }
}

}  // namespace gofann
