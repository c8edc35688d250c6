/*
 * gofann_oracle.c — TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's (putatio13/GO-FANN) filtered-ANN search
 * path, used as the parity checker for the CUDA library and as the timed CPU
 * baseline.  Nothing in the product links or calls this file: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
 * load it.  Every function cites the reference file:line it restates.
 *
 * It consumes the same descriptor structs as the C ABI (include/gofann.h),
 * holding HOST pointers here.
 *
 * Floating-point order is pinned explicitly: every multiply-add that nvcc
 * contracts in the reference (`acc += a * b`) is written as fmaf(), and warp
 * reductions are replayed as the xor butterfly 16,8,4,2,1 over the 32 lane
 * partials.  Build with -ffp-contract=off so the compiler adds no other FMA.
 */
#include "gofann_oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define KW 32
#define HASH_CAP GOFANN_HASH_CAPACITY
#define U32MAX 0xffffffffu
#define POOL_USED 0x80000000u

/* ------------------------------------------------------------- helpers */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* Lane-0 value of the xor butterfly `v += shfl_xor(v, off)` for off =
 * 16,8,4,2,1 (backend_pq.cu:4182-4185, 4716-4721). */
float oracle_warp_sum(const float* lanes)
{
    float v[KW];
    for (int i = 0; i < KW; ++i) v[i] = lanes[i];
    for (int off = KW / 2; off > 0; off >>= 1) {
        float nv[KW];
        for (int i = 0; i < KW; ++i) nv[i] = v[i] + v[i ^ off];
        memcpy(v, nv, sizeof(v));
    }
    return v[0];
}

/* ----------------------------------------------------------------- PQ */

/* computePQTable, backend_pq.cu:1999-2022 (one lane per centroid; per
 * element diff = q - c then `distance += diff*diff` contracted to fma). */
void oracle_pq_build_lut(const float* queries, uint32_t n, uint32_t dim, const float* centroids,
                         uint32_t pq_dim, float* lut)
{
    const uint32_t w = dim / pq_dim;
    for (uint32_t q = 0; q < n; ++q) {
        const float* qv = queries + (size_t)q * dim;
        float* out = lut + (size_t)q * pq_dim * GOFANN_PQ_CENTROIDS;
        for (uint32_t m = 0; m < pq_dim; ++m) {
            for (uint32_t c = 0; c < GOFANN_PQ_CENTROIDS; ++c) {
                float acc = 0.0f;
                for (uint32_t d = 0; d < w; ++d) {
                    const float diff = qv[m * w + d] - centroids[(size_t)c * dim + m * w + d];
                    acc = fmaf(diff, diff, acc);
                }
                out[m * GOFANN_PQ_CENTROIDS + c] = acc;
            }
        }
    }
}

/* ADC in the warp order of backend_pq.cu:4711-4725: lane j accumulates
 * subspaces j, j+32, ... starting from 0, then the butterfly. */
float oracle_pq_adc_one(const float* lut_row, uint32_t pq_dim, const uint8_t* code)
{
    float lanes[KW];
    for (int j = 0; j < KW; ++j) {
        float acc = 0.0f;
        for (uint32_t m = (uint32_t)j; m < pq_dim; m += KW)
            acc = acc + lut_row[m * GOFANN_PQ_CENTROIDS + code[m]];
        lanes[j] = acc;
    }
    return oracle_warp_sum(lanes);
}

void oracle_pq_adc(const float* lut, uint32_t pq_dim, const uint8_t* codes,
                   const uint32_t* pair_row, const uint32_t* pair_sample, uint32_t n_pairs,
                   float* out)
{
    for (uint32_t i = 0; i < n_pairs; ++i)
        out[i] = oracle_pq_adc_one(lut + (size_t)pair_row[i] * pq_dim * GOFANN_PQ_CENTROIDS,
                                   pq_dim, codes + (size_t)pair_sample[i] * pq_dim);
}

/* Posting-scan distance: sequential over subspaces (backend_pq.cu:2101-2104). */
static float pq_seq_dist(const float* lut_row, uint32_t pq_dim, const uint8_t* code)
{
    float d = 0.0f;
    for (uint32_t m = 0; m < pq_dim; ++m) d = d + lut_row[m * GOFANN_PQ_CENTROIDS + code[m]];
    return d;
}

/* Nearest centroid per subspace, squared L2 with the LUT's fma order, lowest
 * centroid index on ties (pq_builder.cu:125-151 semantics; the oracle of
 * tests/native/quantization_smoke.py:35-41 checks codes = nearest centres). */
void oracle_pq_encode(const float* vectors, uint32_t n, uint32_t dim, const float* centroids,
                      uint32_t pq_dim, uint8_t* codes)
{
    const uint32_t w = dim / pq_dim;
    for (uint32_t i = 0; i < n; ++i) {
        const float* x = vectors + (size_t)i * dim;
        for (uint32_t m = 0; m < pq_dim; ++m) {
            float best = INFINITY;
            uint32_t best_c = 0;
            for (uint32_t c = 0; c < GOFANN_PQ_CENTROIDS; ++c) {
                float acc = 0.0f;
                for (uint32_t d = 0; d < w; ++d) {
                    const float diff = x[m * w + d] - centroids[(size_t)c * dim + m * w + d];
                    acc = fmaf(diff, diff, acc);
                }
                if (acc < best) { best = acc; best_c = c; }
            }
            codes[(size_t)i * pq_dim + m] = (uint8_t)best_c;
        }
    }
}

/* ------------------------------------------------------------- RaBitQ */

/* quantize_rabitq_queries_int8_kernel, backend_rabitq.cu:2931-2964 (max is
 * order independent; IEEE division; __float2int_rn = round half even) and
 * the k1xsumq factor of compute_rabitq_query_factors_kernel (2898-2929),
 * whose sum is replayed in the library's order: 256 thread-strided partials
 * then a shared-memory tree halving 128..1. */
void oracle_rabitq_quantize(const float* rotated, uint32_t n, uint32_t padded_dim, int8_t* q8,
                            float* scale_out, float* k1_out)
{
    for (uint32_t q = 0; q < n; ++q) {
        const float* src = rotated + (size_t)q * padded_dim;
        float mx = 0.0f;
        for (uint32_t d = 0; d < padded_dim; ++d) mx = fmaxf(mx, fabsf(src[d]));
        const float scale = mx > 0.0f ? mx / 127.0f : 1.0f;
        scale_out[q] = scale;
        for (uint32_t d = 0; d < padded_dim; ++d) {
            long v = lrintf(src[d] / scale);
            if (v < -127) v = -127;
            if (v > 127) v = 127;
            q8[(size_t)q * padded_dim + d] = (int8_t)v;
        }
        float part[256];
        for (int t = 0; t < 256; ++t) {
            float s = 0.0f;
            for (uint32_t d = (uint32_t)t; d < padded_dim; d += 256) s = s + src[d];
            part[t] = s;
        }
        for (int stride = 128; stride > 0; stride >>= 1)
            for (int t = 0; t < stride; ++t) part[t] = part[t] + part[t + stride];
        k1_out[q] = part[0] * -0.5f;
    }
}

/* Integer part of the 1-bit estimator: sum of q8[d] over set bits, bits
 * MSB-first in little-endian uint32 words (rabitq_dp4a_binary_dot_lane<true>
 * with the nibble masks, backend_rabitq.cu:204-209, 3070-3098). */
int32_t oracle_rabitq_ip(const uint8_t* code, const int8_t* q8, uint32_t padded_dim)
{
    int32_t acc = 0;
    for (uint32_t d = 0; d < padded_dim; ++d) {
        const uint32_t word = (uint32_t)code[(d / 32) * 4] | ((uint32_t)code[(d / 32) * 4 + 1] << 8) |
                              ((uint32_t)code[(d / 32) * 4 + 2] << 16) |
                              ((uint32_t)code[(d / 32) * 4 + 3] << 24);
        if ((word >> (31 - d % 32)) & 1u) acc += q8[d];
    }
    return acc;
}

/* Combine step of score_rabitq_code_device (backend_rabitq.cu:3185-3192):
 * short_ip = float(ip) * scale feeds only `short_ip + k1xsumq`, and the
 * product f_rescale * (...) only the final add, so both mul+add pairs are
 * pinned as contracted:  fma(f_rescale, fma(float(ip), scale, k1), f_add + gdist). */
float oracle_rabitq_combine(int32_t ip, float scale, float k1, float f_add, float f_rescale,
                            float gdist)
{
    const float t = fmaf((float)ip, scale, k1);
    return fmaf(f_rescale, t, f_add + gdist);
}

static float rabitq_est(const gofann_codes* c, const gofann_prepared* p, uint32_t row,
                        uint32_t sample, int32_t* ip_out)
{
    const uint32_t code_bytes = c->padded_dim / 8;
    const int32_t ip = oracle_rabitq_ip(c->rq_codes + (size_t)sample * code_bytes,
                                        p->rq_q8 + (size_t)row * c->padded_dim, c->padded_dim);
    if (ip_out) *ip_out = ip;
    const uint32_t anchor = c->rq_anchor_ids[sample];
    return oracle_rabitq_combine(ip, p->rq_scale[row], p->rq_k1xsumq[row],
                                 c->rq_factors[(size_t)sample * 3],
                                 c->rq_factors[(size_t)sample * 3 + 1],
                                 p->rq_centroid_dist[(size_t)row * c->num_anchors + anchor]);
}

void oracle_rabitq_score(const gofann_codes* c, const gofann_prepared* p,
                         const uint32_t* pair_row, const uint32_t* pair_sample, uint32_t n_pairs,
                         float* out, int32_t* ip_out)
{
    for (uint32_t i = 0; i < n_pairs; ++i)
        out[i] = rabitq_est(c, p, pair_row[i], pair_sample[i], ip_out ? ip_out + i : NULL);
}

/* RaBitQ 1-bit encoding given rotation-applied residuals (quantizer_gpu_fast.cu:180-270,
 * binarise quantizer_gpu.cu:166-170, MSB-first pack 31-46): bit = r > 0,
 * xu = bit - 0.5, f_add = |r|^2 + 2|r|^2 (c.xu)/(r.xu), f_rescale =
 * -2|r|^2/(r.xu), f_err = 2*1.9*|r|*sqrt(max(0,(|r|^2|xu|^2/(r.xu)^2-1)/(P-1))).
 * Sums are sequential in double here; the library encoder is tolerance-checked. */
void oracle_rabitq_encode(const float* residual, const float* rotated_centroid, uint32_t n,
                          uint32_t padded_dim, const uint32_t* anchor_ids, uint8_t* codes,
                          float* factors)
{
    const uint32_t code_bytes = padded_dim / 8;
    for (uint32_t i = 0; i < n; ++i) {
        const float* r = residual + (size_t)i * padded_dim;
        const float* c = rotated_centroid + (size_t)anchor_ids[i] * padded_dim;
        uint8_t* code = codes + (size_t)i * code_bytes;
        memset(code, 0, code_bytes);
        double rr = 0, rxu = 0, cxu = 0, xuxu = 0;
        for (uint32_t d = 0; d < padded_dim; ++d) {
            const int bit = r[d] > 0.0f;
            const double xu = bit ? 0.5 : -0.5;
            rr += (double)r[d] * r[d];
            rxu += (double)r[d] * xu;
            cxu += (double)c[d] * xu;
            xuxu += xu * xu;
            if (bit) {
                const uint32_t word = d / 32, bitpos = 31 - d % 32;
                code[word * 4 + bitpos / 8] |= (uint8_t)(1u << (bitpos % 8));
            }
        }
        float* f = factors + (size_t)i * 3;
        if (rxu == 0.0) rxu = 1e-30;
        f[0] = (float)(rr + 2.0 * rr * cxu / rxu);
        f[1] = (float)(-2.0 * rr / rxu);
        double t = (rr * xuxu / (rxu * rxu) - 1.0) / (double)(padded_dim - 1);
        if (t < 0) t = 0;
        f[2] = (float)(2.0 * 1.9 * sqrt(rr) * sqrt(t));
    }
}

/* The device encoder's FP32 arithmetic (gofann_rabitq_encode): 32 lane
 * partials over dimensions l, l+32, ..., an xor butterfly, the factor
 * formulas left to right; code word w = dimensions 32w..32w+31 MSB first
 * (the RaBitQ quantizer, quantizer_gpu_fast.cu:180-270, packing
 * quantizer_gpu.cu:31-46). */
void oracle_rabitq_encode_f32(const float* residual, const float* rotated_centroid, uint32_t n,
                              uint32_t padded_dim, const uint32_t* anchor_ids, uint32_t* codes, float* factors)
{
    const uint32_t words = padded_dim / 32;
    for (uint32_t i = 0; i < n; ++i) {
        const float* r = residual + (size_t)i * padded_dim;
        const float* c = rotated_centroid + (size_t)anchor_ids[i] * padded_dim;
        float rr[32], rxu[32], cxu[32];
        for (int l = 0; l < 32; ++l) rr[l] = rxu[l] = cxu[l] = 0.0f;
        for (uint32_t w = 0; w < words; ++w) {
            uint32_t word = 0;
            for (int l = 0; l < 32; ++l) {
                const uint32_t d = w * 32 + (uint32_t)l;
                const float x = r[d];
                const int bit = x > 0.0f;
                const float xu = bit ? 0.5f : -0.5f;
                rr[l] = fmaf(x, x, rr[l]);
                rxu[l] = rxu[l] + x * xu;
                cxu[l] = cxu[l] + c[d] * xu;
                if (bit) word |= 0x80000000u >> l;
            }
            codes[(size_t)i * words + w] = word;
        }
        for (int off = 16; off > 0; off >>= 1) {
            float nrr[32], nrxu[32], ncxu[32];
            for (int l = 0; l < 32; ++l) {
                nrr[l] = rr[l] + rr[l ^ off];
                nrxu[l] = rxu[l] + rxu[l ^ off];
                ncxu[l] = cxu[l] + cxu[l ^ off];
            }
            memcpy(rr, nrr, sizeof rr);
            memcpy(rxu, nrxu, sizeof rxu);
            memcpy(cxu, ncxu, sizeof cxu);
        }
        const float R = rr[0], C = cxu[0];
        float X = rxu[0];
        const float xuxu = (float)padded_dim * 0.25f;
        if (X == 0.0f) X = 1e-30f;
        float* f = factors + (size_t)i * 3;
        f[0] = R + ((2.0f * R) * C) / X;
        f[1] = (-2.0f * R) / X;
        float t = ((R * xuxu) / (X * X) - 1.0f) / (float)(padded_dim - 1);
        if (!(t > 0.0f)) t = 0.0f;
        f[2] = (3.8f * sqrtf(R)) * sqrtf(t);
    }
}

/* ------------------------------------------------------- visited hash */
/* native_visited_hash.cuh:11-61 */
static uint32_t hash_code(uint32_t v)
{
    const uint64_t mixed = (uint64_t)v ^ ((uint64_t)(v >> 16) * 0x4bcb391f924ed183ULL) ^
                           0xa0ab69ccd854fc0aULL;
    return (uint32_t)(mixed % HASH_CAP);
}
int oracle_hash_test(const uint32_t* t, uint32_t v)
{
    uint32_t s = hash_code(v);
    for (int p = 0; p < HASH_CAP; ++p) {
        if (t[s] == U32MAX) return 0;
        if (t[s] == v) return 1;
        s = (s + 1) % HASH_CAP;
    }
    return 0;
}
/* returns 0 inserted, 1 existing, 2 full (silently dropped) */
int oracle_hash_add(uint32_t* t, uint32_t v)
{
    uint32_t s = hash_code(v);
    for (int p = 0; p < HASH_CAP; ++p) {
        if (t[s] == v) return 1;
        if (t[s] == U32MAX) { t[s] = v; return 0; }
        s = (s + 1) % HASH_CAP;
    }
    return 2;
}

/* ------------------------------------------------ symmetric min-max heap */
/* include/smmh2.h:8-148.  Entries compare by `first` only. */
typedef struct { float first; uint32_t second; float base; } fpair;

static void fswap(fpair* a, fpair* b) { fpair t = *a; *a = *b; *b = t; }

static int smmh_adjust_sibling(fpair* h, int y, int size)
{
    if (y & 1) {
        const int s = y + 1;
        if (s >= size) return y;
        if (h[y].first > h[s].first) { fswap(&h[y], &h[s]); return s; }
    } else {
        const int s = y - 1;
        if (h[y].first < h[s].first) { fswap(&h[y], &h[s]); return s; }
    }
    return y;
}
static int smmh_adjust_grandparent(fpair* h, int y)
{
    if (y <= 2) return y;
    const int g = (y - 3) >> 2;
    const int gl = 2 * g + 1, gr = 2 * g + 2;
    if (h[gl].first > h[y].first) { fswap(&h[gl], &h[y]); return gl; }
    if (h[gr].first < h[y].first) { fswap(&h[gr], &h[y]); return gr; }
    return y;
}
void oracle_smmh_insert(fpair* h, int* size, fpair e)
{
    int y = *size;
    h[(*size)++] = e;
    for (;;) {
        y = smmh_adjust_sibling(h, y, *size);
        const int x = smmh_adjust_grandparent(h, y);
        if (x == y) break;
        y = x;
    }
}
static int smmh_adjust_grandchild(fpair* h, int y, int size)
{
    if (y & 1) {
        if (2 * y + 1 >= size) return y;
        const int cl = 2 * y + 1, cr = 2 * (y + 1) + 1;
        int c = cl;
        if (cr < size && h[cr].first < h[cl].first) c = cr;
        if (h[c].first < h[y].first) { fswap(&h[c], &h[y]); return c; }
    } else {
        const int cl = 2 * (y - 1) + 2, cr = 2 * y + 2;
        if (cl >= size) return y;
        int c = cl;
        if (cr < size && h[cr].first > h[cl].first) c = cr;
        if (h[c].first > h[y].first) { fswap(&h[c], &h[y]); return c; }
    }
    return y;
}
static void smmh_deletion(fpair* h, int idx, int* size)
{
    h[idx] = h[--(*size)];
    int y = idx;
    for (;;) {
        smmh_adjust_sibling(h, y, *size);
        const int x = smmh_adjust_grandchild(h, y, *size);
        if (x == y) break;
        y = x;
    }
}
fpair oracle_smmh_pop_max(fpair* h, int* size)
{
    fpair r = h[2];
    smmh_deletion(h, 2, size);
    return r;
}
fpair oracle_smmh_pop_min(fpair* h, int* size)
{
    fpair r = h[1];
    smmh_deletion(h, 1, size);
    return r;
}

/* ------------------------------------------------------ binary max heap */
/* include/bin_heap.h:6-16,39-66, generic over an entry with a float key. */
typedef struct { float first; uint32_t second; } rpair;                /* ResultPair */
typedef struct { float first; uint32_t pad; uint64_t second; } spair; /* stop pair */

#define DEFINE_BIN_HEAP(T, NAME)                                                        \
    static void NAME##_push(T* b, int n)                                                \
    {                                                                                   \
        int now = n - 1;                                                                \
        int parent = (now - 1) / 2;                                                     \
        while (now > 0 && b[parent].first < b[now].first) {                             \
            T t = b[now]; b[now] = b[parent]; b[parent] = t;                            \
            now = parent; parent = (now - 1) / 2;                                       \
        }                                                                               \
    }                                                                                   \
    static T NAME##_pop(T* b, int n)                                                    \
    {                                                                                   \
        T ret = b[0];                                                                   \
        const int len = n - 1;                                                          \
        if (len <= 0) return ret;                                                       \
        b[0] = b[n - 1];                                                                \
        int now = 0;                                                                    \
        while (now * 2 + 1 < len) {                                                     \
            const int l = now * 2 + 1, r = now * 2 + 2;                                 \
            int nx = l;                                                                 \
            if (r < len && b[l].first < b[r].first) nx = r;                             \
            if (!(b[now].first < b[nx].first)) break;                                   \
            T t = b[now]; b[now] = b[nx]; b[nx] = t;                                    \
            now = nx;                                                                   \
        }                                                                               \
        return ret;                                                                     \
    }
DEFINE_BIN_HEAP(rpair, rheap)
DEFINE_BIN_HEAP(spair, sheap)

void oracle_rheap_push(float* firsts, uint32_t* seconds, int n)
{
    rpair b[GOFANN_MAX_RESULT_WIDTH + 1];
    for (int i = 0; i < n; ++i) { b[i].first = firsts[i]; b[i].second = seconds[i]; }
    rheap_push(b, n);
    for (int i = 0; i < n; ++i) { firsts[i] = b[i].first; seconds[i] = b[i].second; }
}
void oracle_rheap_pop(float* firsts, uint32_t* seconds, int n, float* out_first, uint32_t* out_second)
{
    rpair b[GOFANN_MAX_RESULT_WIDTH + 1];
    for (int i = 0; i < n; ++i) { b[i].first = firsts[i]; b[i].second = seconds[i]; }
    rpair r = rheap_pop(b, n);
    for (int i = 0; i < n; ++i) { firsts[i] = b[i].first; seconds[i] = b[i].second; }
    *out_first = r.first; *out_second = r.second;
}

/* --------------------------------------------- (dist,id) shortlist heap */
/* search/common/posting_shortlist_heap.cuh:14-99 */
static int pair_is_worse(float ld, uint32_t li, float rd, uint32_t ri)
{
    return ld > rd || (ld == rd && li > ri);
}
static void sl_sift_down(float* d, uint32_t* id, int n, int root)
{
    for (;;) {
        const int l = root * 2 + 1;
        if (l >= n) break;
        const int r = l + 1;
        int w = l;
        if (r < n && pair_is_worse(d[r], id[r], d[l], id[l])) w = r;
        if (!pair_is_worse(d[w], id[w], d[root], id[root])) break;
        float td = d[root]; uint32_t ti = id[root];
        d[root] = d[w]; id[root] = id[w]; d[w] = td; id[w] = ti;
        root = w;
    }
}
int oracle_sl_can_enter(float dist, uint32_t id, const float* d, const uint32_t* ids, int k)
{
    return id != U32MAX && k > 0 && pair_is_worse(d[0], ids[0], dist, id);
}
void oracle_sl_insert(float dist, uint32_t id, float* d, uint32_t* ids, int k)
{
    if (!oracle_sl_can_enter(dist, id, d, ids, k)) return;
    d[0] = dist; ids[0] = id;
    sl_sift_down(d, ids, k, 0);
}
void oracle_sl_sort(float* d, uint32_t* ids, int k)
{
    for (int n = k; n > 1; --n) {
        const int tail = n - 1;
        float td = d[0]; uint32_t ti = ids[0];
        d[0] = d[tail]; ids[0] = ids[tail]; d[tail] = td; ids[tail] = ti;
        sl_sift_down(d, ids, tail, 0);
    }
}

/* ----------------------------------------------------------- predicates */

static int csr_contains(const gofann_attrs* a, uint32_t sample, uint32_t label)
{
    /* gpu_predicate_index.cuh:59-84 (membership in the sorted sample row) */
    const uint64_t b = a->label_indptr[sample], e = a->label_indptr[sample + 1];
    for (uint64_t i = b; i < e; ++i) {
        const uint32_t l = a->label_indices[i];
        if (l >= label) return l == label;
    }
    return 0;
}
static int range_match(uint32_t mode, float lo, float hi, float v)
{
    switch (mode) {  /* range_filter.cuh:28-45, gpu_predicate_index.cuh:100-108 */
    case 0: return 1;
    case 1: return v > lo;
    case 2: return v < hi;
    case 3: return v >= lo && v < hi;
    default: return 0;
    }
}
int oracle_pred_enabled(const gofann_routes* r, uint32_t route)
{
    if (!r->pred_offsets) return 0;
    return r->pred_enabled ? r->pred_enabled[route] != 0 : 1;
}
/* Levenshtein distance by the textbook dynamic programme (Wagner and
 * Fischer, J. ACM 21(1), 1974), two rows. */
uint32_t oracle_levenshtein(const uint8_t* p, uint32_t m, const uint8_t* t, uint32_t n)
{
    uint32_t* prev = (uint32_t*)malloc(sizeof(uint32_t) * (n + 1));
    uint32_t* cur = (uint32_t*)malloc(sizeof(uint32_t) * (n + 1));
    for (uint32_t j = 0; j <= n; ++j) prev[j] = j;
    for (uint32_t i = 1; i <= m; ++i) {
        cur[0] = i;
        for (uint32_t j = 1; j <= n; ++j) {
            uint32_t v = prev[j - 1] + (p[i - 1] != t[j - 1]);
            if (prev[j] + 1 < v) v = prev[j] + 1;
            if (cur[j - 1] + 1 < v) v = cur[j - 1] + 1;
            cur[j] = v;
        }
        uint32_t* tmp = prev; prev = cur; cur = tmp;
    }
    const uint32_t d = prev[n];
    free(prev);
    free(cur);
    return d;
}

/* String and integer atoms of clause ci (gofann_clause_ext): exact string
 * equality, Levenshtein distance <= max_edits, int64 ranges in the float
 * atom's modes. */
static int ext_atoms_match(const gofann_routes* r, const gofann_attrs* a, uint32_t ci, uint32_t sample)
{
    const gofann_clause_ext x = r->pred_ext[ci];
    for (uint32_t j = x.int_begin; j < x.int_end; ++j) {
        const gofann_int_atom at = r->pred_ints[j];
        if (at.mode == 0) continue;
        if (!a->int_values || at.dimension >= a->int_count) return 0;
        const int64_t v = a->int_values[(size_t)sample * a->int_count + at.dimension];
        int ok = 0;
        if (at.mode == 1) ok = v > at.lower;
        else if (at.mode == 2) ok = v < at.upper;
        else if (at.mode == 3) ok = v >= at.lower && v < at.upper;
        if (!ok) return 0;
    }
    if (x.string_begin == x.string_end) return 1;
    if (!a->string_offsets) return 0;
    const uint8_t* t = a->string_bytes + a->string_offsets[sample];
    const uint32_t n = (uint32_t)(a->string_offsets[sample + 1] - a->string_offsets[sample]);
    for (uint32_t j = x.string_begin; j < x.string_end; ++j) {
        const gofann_string_atom at = r->pred_strings[j];
        const uint8_t* q = r->pred_string_bytes + at.offset;
        if (at.kind == GOFANN_STRING_EXACT) {
            if (n != at.length || memcmp(t, q, n) != 0) return 0;
        } else {
            if (at.length > GOFANN_FUZZY_MAX_LENGTH) return 0;
            if (oracle_levenshtein(q, at.length, t, n) > at.max_edits) return 0;
        }
    }
    return 1;
}

/* gpu_predicate::matches with clauses, gpu_predicate_index.cuh:109-136,
 * then each clause's string and integer atoms */
int oracle_pred_matches(const gofann_routes* r, const gofann_attrs* a, uint32_t route,
                        uint32_t sample)
{
    if (sample >= a->n_samples) return 0;
    for (uint32_t i = r->pred_offsets[route]; i < r->pred_offsets[route + 1]; ++i) {
        const gofann_clause c = r->clauses[i];
        int pass = 1;
        for (uint32_t j = c.label_begin; pass && j < c.label_end; ++j)
            pass = csr_contains(a, sample, r->pred_handles[j]);
        for (uint32_t j = c.range_begin; pass && j < c.range_end; ++j) {
            const gofann_range_atom at = r->pred_ranges[j];
            pass = a->range_values && at.dimension < a->range_count &&
                   range_match(at.mode, at.lower, at.upper,
                               a->range_values[(size_t)sample * a->range_count + at.dimension]);
        }
        if (pass && r->pred_ext) pass = ext_atoms_match(r, a, i, sample);
        if (pass) return 1;
    }
    return 0;
}
/* resident_pq_labels_match, backend_pq.cu:3934-3965 */
int oracle_labels_match(const gofann_routes* r, const gofann_attrs* a, uint32_t route,
                        uint32_t sample)
{
    if (!r->qlabel_indptr) return 1;
    const uint32_t primary = r->primary_label ? r->primary_label[route] : U32MAX;
    for (uint64_t p = r->qlabel_indptr[route]; p < r->qlabel_indptr[route + 1]; ++p) {
        const uint32_t l = r->qlabel_indices[p];
        if (l == primary) continue;
        uint64_t lo = a->label_indptr[sample], hi = a->label_indptr[sample + 1];
        const uint64_t end = hi;
        while (lo < hi) {
            const uint64_t mid = lo + ((hi - lo) >> 1);
            if (a->label_indices[mid] < l) lo = mid + 1; else hi = mid;
        }
        if (lo == end || a->label_indices[lo] != l) return 0;
    }
    return 1;
}
/* range_filter.cuh:47-98 */
static uint32_t count_active(const gofann_routes* r, uint32_t route)
{
    if (!r->range_modes) return 0;
    uint32_t n = 0;
    for (uint32_t i = 0; i < r->range_count; ++i)
        if (r->range_modes[(size_t)route * r->range_count + i] != 0) ++n;
    return n;
}
static uint32_t count_matching(const gofann_routes* r, const gofann_attrs* a, uint32_t route,
                               uint32_t sample)
{
    if (!r->range_modes || !r->range_lower || !r->range_upper) return 0;
    uint32_t n = 0;
    for (uint32_t i = 0; i < r->range_count; ++i) {
        const size_t qf = (size_t)route * r->range_count + i;
        const uint8_t mode = r->range_modes[qf];
        if (mode == 0) continue;
        if (!a->range_values) return 0;
        if (range_match(mode, r->range_lower[qf], r->range_upper[qf],
                        a->range_values[(size_t)sample * r->range_count + i]))
            ++n;
    }
    return n;
}

/* gpu_predicate::priority, gpu_predicate_index.cuh:161-166 */
static float pred_priority(float base, float penalty, int pass)
{
    if (pass || penalty == 0.0f || !isfinite(base) || base == FLT_MAX) return base;
    if (base > FLT_MAX - penalty) return FLT_MAX;
    return base + penalty;
}

/* adaptive_early_stop_limit / early_stop_reached, backend_pq.cu:2822-2873 */
static int adaptive_limit(int queue_limit, int expanded, int pass, int stop_width)
{
    const int queue_base = queue_limit > 1 ? queue_limit : 1;
    int base_limit = (queue_base * 1 + 2 - 1) / 2;
    const int min_base = stop_width > 0 ? stop_width * 2 : 1;
    base_limit = base_limit > min_base ? base_limit : min_base;
    const int denom = (expanded + 16) > 1 ? (expanded + 16) : 1;
    const int pw = pass + 8;
    const int pest = pw < denom ? pw : denom;
    const int rej = (denom - pest) > 0 ? (denom - pest) : 0;
    const int64_t num = (int64_t)queue_limit * 1 * rej;
    int extra = (int)((num + (2 * denom - 1)) / (2 * denom));
    extra = extra > 0 ? extra : 0;
    extra = extra < 32 ? extra : 32;
    return base_limit + extra;
}
static int early_stop(int mode, int bad, int fixed, int queue_limit, int expanded, int pass,
                      int stop_width)
{
    if (mode == GOFANN_EARLY_STOP_OFF) return 0;
    if (mode == GOFANN_EARLY_STOP_ADAPTIVE)
        return bad >= adaptive_limit(queue_limit, expanded, pass, stop_width);
    return bad >= fixed;
}

/* ---------------------------------------------------------- traversal */

/* pickup_next_unused_from_native_frontier<kCooperative=true>,
 * backend_pq.cu:844-893 (RaBitQ twin backend_rabitq.cu:924-970): lane l
 * scans entries l+1, l+33, ... and keeps the first unused entry of smallest
 * `first`; a shfl_down tree (offsets 16..1) then merges lane l+off into lane
 * l, replacing lane l's candidate only by a strictly smaller distance.  The
 * source also replaces on equal distances when the other index is smaller,
 * but the reference compiled for sm_100a (nvcc 12.9, run on a B200 through
 * oracle/ref_kernels.cu on 600 tie-heavy frontiers and 8 traversal cases,
 * tests/golden/reference_pq_kernel.npz) never does: on ties the receiving
 * lane keeps its candidate.  This restates that observed behaviour lane by
 * lane; the result is lane 0's candidate, which lane 0 copies and marks. */
static int pickup(fpair* f, int size, fpair* out)
{
    int bi[32];
    float bd[32];
    for (int l = 0; l < 32; ++l) {
        bi[l] = -1;
        bd[l] = FLT_MAX;
        for (int i = l + 1; i < size; i += 32) {
            if (f[i].second & POOL_USED) continue;
            if (bi[l] < 0 || f[i].first < bd[l]) { bi[l] = i; bd[l] = f[i].first; }
        }
    }
    for (int off = 16; off > 0; off >>= 1) {
        int oi[32];
        float od[32];
        for (int l = 0; l < 32; ++l) {  /* shfl_down: lanes past the end read their own value */
            const int src = l + off < 32 ? l + off : l;
            oi[l] = bi[src];
            od[l] = bd[src];
        }
        for (int l = 0; l < 32; ++l)
            if (oi[l] >= 0 && (bi[l] < 0 || od[l] < bd[l])) { bi[l] = oi[l]; bd[l] = od[l]; }
    }
    const int best = bi[0];
#ifdef ORACLE_DEBUG_PICKUP
    printf("PICK size=%d idx=%d row=%u first=%.9g\n", size, best,
           best >= 0 ? (f[best].second & ~POOL_USED) : 0xffffffffu, best >= 0 ? (double)f[best].first : 0.0);
#endif
    if (best < 0) return 0;
    *out = f[best];
    f[best].second |= POOL_USED;
    return 1;
}

/* The entry pickup() takes from a frontier of `size` entries (index 0
 * unused; vals carry the used bit), or -1; nothing is modified. */
int oracle_pickup_index(const float* keys, const uint32_t* vals, int size)
{
    fpair* f = (fpair*)calloc((size_t)(size > 1 ? size : 1), sizeof(fpair));
    for (int i = 0; i < size; ++i) { f[i].first = keys[i]; f[i].second = vals[i]; f[i].base = keys[i]; }
    fpair out;
    int idx = -1;
    if (pickup(f, size, &out)) idx = (int)(out.second & ~POOL_USED);
    free(f);
    return idx;
}

static float route_distance(const gofann_codes* c, const gofann_prepared* p, int scorer,
                            uint32_t row, uint32_t sample)
{
    if (scorer == GOFANN_SCORER_PQ)
        return oracle_pq_adc_one(p->pq_lut + (size_t)row * c->pq_dim * GOFANN_PQ_CENTROIDS, c->pq_dim,
                                 c->pq_codes + (size_t)sample * c->pq_dim);
    return rabitq_est(c, p, row, sample, NULL);
}

/*
 * One route of the device-resident traversal loop, run_pq_search_one_block
 * (backend_pq.cu:3988-5013) with kDeviceResident, cooperative pickup, no
 * static prefetch and unit filter bonuses; the RaBitQ loop
 * (backend_rabitq.cu:3593-4292) has the same frontier/stop/top-k logic with
 * the estimator as the scorer.
 */
static void search_one(const gofann_graph* g, const gofann_attrs* a, const gofann_codes* c,
                       const gofann_prepared* p, const gofann_routes* r,
                       const gofann_search_params* sp, uint32_t route, uint32_t* out_ids,
                       float* out_d, int32_t* out_steps, uint32_t* counters, uint32_t* hash,
                       fpair* frontier, rpair* topk, uint32_t* trace, uint32_t trace_width)
{
    const int QS = sp->queue_size, SW = sp->stop_width, RW = sp->result_width;
    const uint32_t row = r->query_row[route];
    const uint32_t group = r->group_id[route];
    const uint32_t label_offset = g->label_offset[group];
    const uint64_t qbit = r->filter_bits ? r->filter_bits[route] : ~0ull;
    const uint32_t active = count_active(r, route);
    const uint32_t begin_id = r->start_local[route];
    const int pred_on = oracle_pred_enabled(r, route);
    const int bias = sp->predicate_bias != 0;
    uint32_t n_expanded = 0, n_dist = 0, n_probe = 0, n_admit = 0;

    for (int i = 0; i < HASH_CAP; ++i) hash[i] = U32MAX;

    const uint32_t begin_sample = g->row_to_sample[label_offset + begin_id];
    const float start_distance = route_distance(c, p, sp->scorer, row, begin_sample);
    ++n_dist;
    float penalty = 0.0f;
    if (bias) {
        const double wide = (double)sp->alpha * fmax((double)fabsf(start_distance), 1e-6);
        penalty = isfinite(wide) ? (float)fmin(wide, (double)FLT_MAX) : 0.0f;
    }

    int heap_size = 1;
    spair stop_topk[GOFANN_MAX_TOPK + 1];
    int stop_size = 0, topk_size = 0;
    float stop_worst = -FLT_MAX;
    int finished = 0, exhausted = 0, expanded = 0, passed = 0;
    fpair now, next;
    {
        fpair kp = {start_distance, begin_id, start_distance};
        oracle_smmh_insert(frontier, &heap_size, kp);
        oracle_hash_add(hash, begin_id);
    }
    if (!pickup(frontier, heap_size, &now)) {
        exhausted = 1;
        now.first = FLT_MAX; now.second = U32MAX | POOL_USED; now.base = FLT_MAX;
    }
    uint32_t list[GOFANN_MAX_DEGREE];
    float dist[GOFANN_MAX_DEGREE];
    int step = 0;
    while (step == 0 || heap_size > 1) {
        const uint32_t now_row = now.second & ~POOL_USED;
        ++step;
        int len = 0;
        if (step != 1) {
            const int found = pickup(frontier, heap_size, &next);
            if (!found) {
                exhausted = 1;
                next.first = FLT_MAX; next.second = U32MAX | POOL_USED; next.base = FLT_MAX;
            } else if (stop_size == SW) {
                float pending = next.first;
                if (sp->pending_base_stop && pred_on) {
                    /* gpu_predicate::minimum_pending_base (gpu_predicate_index.cuh:150-160) */
                    float m = FLT_MAX;
                    m = fminf(m, bias ? now.base : now.first);
                    m = fminf(m, bias ? next.base : next.first);
                    for (int i = 1; i < heap_size; ++i)
                        if (!(frontier[i].second & POOL_USED))
                            m = fminf(m, bias ? frontier[i].base : frontier[i].first);
                    pending = m;
                }
                if (sp->early_stop_mode != GOFANN_EARLY_STOP_OFF && stop_worst <= pending)
                    ++finished;
            }
        }
        /* The reference evaluates the filter of `now` and then breaks on an
         * exhausted pool; when `now` is the exhaustion sentinel that filter
         * would read row 0x7fffffff, so the break is taken first here. The
         * outcome is identical: the filter result is unused once breaking. */
        if (exhausted) break;
        const uint32_t grow = label_offset + now_row;
        const int bit_match = g->row_filter_mask ? (g->row_filter_mask[grow] & qbit) != 0
                                                 : qbit != 0;
        const uint32_t sample = g->row_to_sample[grow];
        const uint32_t matched = count_matching(r, a, route, sample);
        const int exact_range = active == 0 || matched == active;
        int nfr = (sp->full_label_check == 0 || oracle_labels_match(r, a, route, sample)) ? 1 : 2;
        if (pred_on) {
            nfr = oracle_pred_matches(r, a, route, sample) ? 1 : 2;
            ++n_probe;
        } else if (!r->route_compiled || !r->route_compiled[route]) {
            nfr = (nfr == 1 && bit_match && exact_range) ? 1 : 2;
        }
        const float current = bias ? now.base : now.first;
        if (exhausted || early_stop(sp->early_stop_mode, finished, sp->finish_limit, QS, expanded,
                                    passed, SW) ||
            (sp->max_steps > 0 && step >= sp->max_steps))
            break;
        if (trace && (uint32_t)expanded < trace_width) trace[expanded] = now_row;
        ++expanded;
        ++n_expanded;
        if (nfr == 1) {
            ++passed;
            rpair te = {current, now_row};
            spair se;
            se.first = current; se.pad = 0;
            se.second = ((uint64_t)f2u(current) << 32) | now_row;
            int improved = 0;
            if (stop_size < SW) {
                stop_topk[stop_size++] = se;
                sheap_push(stop_topk, stop_size);
                improved = 1;
                if (stop_size == 1 || current > stop_worst) stop_worst = current;
            } else if (se.first < stop_topk[0].first) {
                stop_topk[stop_size++] = se;
                sheap_push(stop_topk, stop_size);
                spair removed = sheap_pop(stop_topk, stop_size);
                --stop_size;
                improved = 1;
                const uint32_t removed_bits = (uint32_t)(removed.second >> 32);
                if (current > stop_worst) {
                    stop_worst = current;
                } else if (removed_bits == f2u(stop_worst)) {
                    stop_worst = -FLT_MAX;
                    for (int i = 0; i < stop_size; ++i) {
                        const float pd = u2f((uint32_t)(stop_topk[i].second >> 32));
                        if (pd > stop_worst) stop_worst = pd;
                    }
                }
            }
            if (sp->early_stop_mode == GOFANN_EARLY_STOP_ADAPTIVE && improved) finished = 0;
            if (topk_size < RW) {
                topk[topk_size++] = te;
                rheap_push(topk, topk_size);
            } else if (te.first < topk[0].first) {
                topk[topk_size++] = te;
                rheap_push(topk, topk_size);
                rheap_pop(topk, topk_size);
                --topk_size;
            }
        }
        const uint32_t deg = g->degree < GOFANN_MAX_DEGREE ? g->degree : GOFANN_MAX_DEGREE;
        for (uint32_t i = 0; i < deg; ++i) {
            const uint32_t idx = g->adjacency[(size_t)grow * g->degree + i];
            if (idx == U32MAX) continue;
            if (oracle_hash_test(hash, idx)) continue;
            list[len++] = idx;
        }
        if (exhausted || early_stop(sp->early_stop_mode, finished, sp->finish_limit, QS, expanded,
                                    passed, SW) ||
            (sp->max_steps > 0 && step >= sp->max_steps))
            break;
        for (int i = 0; i < len; ++i) {
            const uint32_t s = g->row_to_sample[label_offset + list[i]];
            dist[i] = route_distance(c, p, sp->scorer, row, s);
        }
        n_dist += (uint32_t)len;
        for (int i = 0; i < len; ++i) {
            fpair kp;
            kp.first = dist[i];
            kp.base = kp.first;
            if (bias && pred_on) {
                const uint32_t s = g->row_to_sample[label_offset + list[i]];
                const int pass = oracle_pred_matches(r, a, route, s);
                ++n_probe;
                kp.first = pred_priority(kp.base, penalty, pass);
            }
            kp.second = list[i];
            if (heap_size >= QS + 1 && frontier[2].first < kp.first) continue;
            oracle_smmh_insert(frontier, &heap_size, kp);
            oracle_hash_add(hash, list[i]);
            ++n_admit;
            if (heap_size >= QS + 2) oracle_smmh_pop_max(frontier, &heap_size);
        }
        if (step == 1) {
            if (!pickup(frontier, heap_size, &next)) {
                exhausted = 1;
                next.first = FLT_MAX; next.second = U32MAX | POOL_USED; next.base = FLT_MAX;
            }
        }
        now = next;
    }

    const int valid = topk_size < RW ? topk_size : RW;
    for (int i = 0; i < RW; ++i) { out_ids[i] = U32MAX; out_d[i] = FLT_MAX; }
    for (int i = 0; i < valid; ++i) {
        rpair res = rheap_pop(topk, topk_size - i);
        const int slot = valid - 1 - i;
        if (res.second == U32MAX) continue;
        out_ids[slot] = g->row_to_sample[label_offset + res.second];
        out_d[slot] = res.first;
    }
    if (trace)
        for (uint32_t i = (uint32_t)expanded; i < trace_width; ++i) trace[i] = U32MAX;
    if (out_steps) *out_steps = step;
    if (counters) {
        counters[0] = n_expanded; counters[1] = n_dist; counters[2] = n_probe; counters[3] = n_admit;
    }
}

typedef struct {
    const gofann_graph* g; const gofann_attrs* a; const gofann_codes* c; const gofann_prepared* p;
    const gofann_routes* r; const gofann_search_params* sp;
    uint32_t* ids; float* d; int32_t* steps; uint32_t* counters;
    uint32_t begin, end, stride;
    uint32_t* trace; uint32_t trace_width;
} search_job;

static void* search_worker(void* arg)
{
    search_job* j = (search_job*)arg;
    const int RW = j->sp->result_width;
    uint32_t* hash = (uint32_t*)malloc(HASH_CAP * sizeof(uint32_t));
    fpair* frontier = (fpair*)malloc((size_t)(j->sp->queue_size + 3) * sizeof(fpair));
    rpair* topk = (rpair*)malloc((size_t)(RW + 2) * sizeof(rpair));
    for (uint32_t route = j->begin; route < j->end; route += j->stride)
        search_one(j->g, j->a, j->c, j->p, j->r, j->sp, route, j->ids + (size_t)route * RW,
                   j->d + (size_t)route * RW, j->steps ? j->steps + route : NULL,
                   j->counters ? j->counters + (size_t)route * 4 : NULL, hash, frontier, topk,
                   j->trace ? j->trace + (size_t)route * j->trace_width : NULL, j->trace_width);
    free(hash); free(frontier); free(topk);
    return NULL;
}

int oracle_beam_search_traced(const gofann_graph* g, const gofann_attrs* a, const gofann_codes* c,
                              const gofann_prepared* p, const gofann_routes* r,
                              const gofann_search_params* sp, uint32_t* ids, float* d, int32_t* steps,
                              uint32_t* counters, int threads, uint32_t* trace, uint32_t trace_width);

int oracle_beam_search(const gofann_graph* g, const gofann_attrs* a, const gofann_codes* c,
                       const gofann_prepared* p, const gofann_routes* r,
                       const gofann_search_params* sp, uint32_t* ids, float* d, int32_t* steps,
                       uint32_t* counters, int threads)
{
    return oracle_beam_search_traced(g, a, c, p, r, sp, ids, d, steps, counters, threads, NULL, 0);
}

int oracle_beam_search_traced(const gofann_graph* g, const gofann_attrs* a, const gofann_codes* c,
                              const gofann_prepared* p, const gofann_routes* r,
                              const gofann_search_params* sp, uint32_t* ids, float* d, int32_t* steps,
                              uint32_t* counters, int threads, uint32_t* trace, uint32_t trace_width)
{
    if (sp->queue_size < 1 || sp->queue_size > GOFANN_MAX_QUEUE || sp->stop_width < 1 ||
        sp->stop_width > GOFANN_MAX_TOPK || sp->result_width < 1 ||
        sp->result_width > GOFANN_MAX_RESULT_WIDTH)
        return GOFANN_ERR_INVALID;
    if (threads < 1) threads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    search_job* jobs = (search_job*)malloc(sizeof(search_job) * (size_t)threads);
    for (int t = 0; t < threads; ++t) {
        search_job j = {g, a, c, p, r, sp, ids, d, steps, counters, (uint32_t)t, r->n_routes,
                        (uint32_t)threads, trace, trace_width};
        jobs[t] = j;
        if (threads == 1) search_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, search_worker, &jobs[t]);
    }
    if (threads > 1)
        for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
    free(th); free(jobs);
    return GOFANN_OK;
}

/* ------------------------------------------------------ posting scan */
/* run_lowfreq_pq_scan_one_block, backend_pq.cu:2046-2134; the RaBitQ scan
 * (backend_rabitq.cu:5396-5493) has the same admission order. */
int oracle_posting_scan(const gofann_codes* c, const gofann_prepared* p, const gofann_attrs* a,
                        const gofann_routes* r, int scorer, const uint32_t* posting_ids,
                        const uint64_t* route_begin, const uint32_t* route_count, int k,
                        int score_first, uint32_t* out_ids, float* out_d)
{
    if (k < 1 || k > GOFANN_MAX_SHORTLIST) return GOFANN_ERR_INVALID;
    for (uint32_t route = 0; route < r->n_routes; ++route) {
        float* bd = out_d + (size_t)route * k;
        uint32_t* bi = out_ids + (size_t)route * k;
        for (int i = 0; i < k; ++i) { bd[i] = FLT_MAX; bi[i] = U32MAX; }
        const uint32_t row = r->query_row[route];
        const int pred_on = oracle_pred_enabled(r, route);
        for (uint32_t i = 0; i < route_count[route]; ++i) {
            const uint32_t s = posting_ids[route_begin[route] + i];
            if (s == U32MAX) continue;
            if (!score_first && pred_on && !oracle_pred_matches(r, a, route, s)) continue;
            const float dist =
                scorer == GOFANN_SCORER_PQ
                    ? pq_seq_dist(p->pq_lut + (size_t)row * c->pq_dim * GOFANN_PQ_CENTROIDS,
                                  c->pq_dim, c->pq_codes + (size_t)s * c->pq_dim)
                    : rabitq_est(c, p, row, s, NULL);
            if (score_first) {
                if (!oracle_sl_can_enter(dist, s, bd, bi, k)) continue;
                if (pred_on && !oracle_pred_matches(r, a, route, s)) continue;
            }
            oracle_sl_insert(dist, s, bd, bi, k);
        }
        oracle_sl_sort(bd, bi, k);
    }
    return GOFANN_OK;
}

/* ----------------------------------------------------------- rerank */

static float f16_decode(uint16_t v)
{
    /* fp16_l2::decode, src/data/fp16_l2.h:20-41 */
    const uint32_t sign = (uint32_t)(v & 0x8000u) << 16;
    uint32_t e = (v >> 10) & 0x1fu, m = v & 0x03ffu, bits;
    if (e == 0) {
        if (m == 0) bits = sign;
        else {
            e = 1;
            while ((m & 0x0400u) == 0) { m <<= 1; --e; }
            bits = sign | ((e + 112u) << 23) | ((m & 0x03ffu) << 13);
        }
    } else if (e == 0x1fu) bits = sign | 0x7f800000u | (m << 13);
    else bits = sign | ((e + 112u) << 23) | (m << 13);
    return u2f(bits);
}

/* Exact L2: uint8 as integer squares (backend_pq.cu:2187-2195, exact in
 * float below 2^24), f32 and f16 sequential `sum += diff*diff` with fma
 * (fp16_l2.h:160-168, dataloader.cpp:2375-2420). */
float oracle_exact_l2(const void* base, int dtype, uint32_t dim, uint32_t sample, const void* query,
                      uint32_t row)
{
    if (dtype == GOFANN_DTYPE_U8) {
        const uint8_t* b = (const uint8_t*)base + (size_t)sample * dim;
        const uint8_t* q = (const uint8_t*)query + (size_t)row * dim;
        int64_t acc = 0;
        for (uint32_t d = 0; d < dim; ++d) {
            const int diff = (int)b[d] - (int)q[d];
            acc += diff * diff;
        }
        return (float)acc;
    }
    const float* q = (const float*)query + (size_t)row * dim;
    float acc = 0.0f;
    if (dtype == GOFANN_DTYPE_F32) {
        const float* b = (const float*)base + (size_t)sample * dim;
        for (uint32_t d = 0; d < dim; ++d) { const float diff = q[d] - b[d]; acc = fmaf(diff, diff, acc); }
    } else {
        const uint16_t* b = (const uint16_t*)base + (size_t)sample * dim;
        for (uint32_t d = 0; d < dim; ++d) {
            const float diff = q[d] - f16_decode(b[d]);
            acc = fmaf(diff, diff, acc);
        }
    }
    return acc;
}

/* highfreq_host_batch_rerank_range, backend_pq.cu:2479-2592: drop sentinel /
 * out-of-range ids, residual label check, duplicates, then top-k by
 * (dist, id) ascending. */
int oracle_rerank(const void* base, int dtype, uint32_t n_samples, uint32_t dim, const void* queries,
                  const gofann_attrs* a, const gofann_routes* r, const uint32_t* cand,
                  uint32_t width, int k, uint32_t* out_ids, float* out_d)
{
    if (k < 1 || k > GOFANN_MAX_TOPK) return GOFANN_ERR_INVALID;
    for (uint32_t route = 0; route < r->n_routes; ++route) {
        const uint32_t row = r->query_row[route];
        float bd[GOFANN_MAX_TOPK];
        uint32_t bi[GOFANN_MAX_TOPK];
        for (int i = 0; i < k; ++i) { bd[i] = FLT_MAX; bi[i] = U32MAX; }
        const uint32_t* cr = cand + (size_t)route * width;
        for (uint32_t i = 0; i < width; ++i) {
            const uint32_t s = cr[i];
            if (s == U32MAX || s >= n_samples) continue;
            int dup = 0;
            for (uint32_t j = 0; j < i; ++j) if (cr[j] == s) { dup = 1; break; }
            if (dup) continue;
            if (a && r->qlabel_indptr && !oracle_labels_match(r, a, route, s)) continue;
            const float dist = oracle_exact_l2(base, dtype, dim, s, queries, row);
            oracle_sl_insert(dist, s, bd, bi, k);
        }
        oracle_sl_sort(bd, bi, k);
        memcpy(out_ids + (size_t)route * k, bi, sizeof(uint32_t) * (size_t)k);
        memcpy(out_d + (size_t)route * k, bd, sizeof(float) * (size_t)k);
    }
    return GOFANN_OK;
}

/* ----------------------------------------------------------- merges */
/* merge_route_results_to_original, rabitq_lowfreq_merge.h:748-815 */
int oracle_route_merge(const uint32_t* ids, const float* d, uint32_t width,
                       const uint32_t* qoff, const uint32_t* qroutes, uint32_t nq, int k,
                       uint32_t* out_ids, float* out_d)
{
    if (k < 1 || k > GOFANN_MAX_TOPK) return GOFANN_ERR_INVALID;
    for (uint32_t q = 0; q < nq; ++q) {
        float bd[GOFANN_MAX_TOPK];
        uint32_t bi[GOFANN_MAX_TOPK];
        for (int i = 0; i < k; ++i) { bd[i] = FLT_MAX; bi[i] = U32MAX; }
        /* unique ids with their minimum distance, then (dist, id) top-k */
        const uint32_t nr = qoff[q + 1] - qoff[q];
        const size_t total = (size_t)nr * width;
        uint32_t* cid = (uint32_t*)malloc(sizeof(uint32_t) * (total + 1));
        float* cd = (float*)malloc(sizeof(float) * (total + 1));
        size_t n = 0;
        for (uint32_t t = qoff[q]; t < qoff[q + 1]; ++t) {
            const uint32_t route = qroutes[t];
            for (uint32_t i = 0; i < width; ++i) {
                const uint32_t s = ids[(size_t)route * width + i];
                if (s == U32MAX) continue;
                const float dist = d[(size_t)route * width + i];
                size_t j = 0;
                for (; j < n; ++j) if (cid[j] == s) break;
                if (j == n) { cid[n] = s; cd[n] = dist; ++n; }
                else if (dist < cd[j]) cd[j] = dist;
            }
        }
        for (size_t j = 0; j < n; ++j) oracle_sl_insert(cd[j], cid[j], bd, bi, k);
        oracle_sl_sort(bd, bi, k);
        memcpy(out_ids + (size_t)q * k, bi, sizeof(uint32_t) * (size_t)k);
        memcpy(out_d + (size_t)q * k, bd, sizeof(float) * (size_t)k);
        free(cid); free(cd);
    }
    return GOFANN_OK;
}

int oracle_shard_merge(const uint32_t* ids, const float* d, uint32_t shards, uint32_t nq, int k,
                       uint32_t* out_ids, float* out_d)
{
    if (k < 1 || k > GOFANN_MAX_TOPK) return GOFANN_ERR_INVALID;
    for (uint32_t q = 0; q < nq; ++q) {
        float bd[GOFANN_MAX_TOPK];
        uint32_t bi[GOFANN_MAX_TOPK];
        for (int i = 0; i < k; ++i) { bd[i] = FLT_MAX; bi[i] = U32MAX; }
        for (uint32_t s = 0; s < shards; ++s)
            for (int i = 0; i < k; ++i) {
                const size_t at = ((size_t)s * nq + q) * k + i;
                oracle_sl_insert(d[at], ids[at], bd, bi, k);
            }
        oracle_sl_sort(bd, bi, k);
        memcpy(out_ids + (size_t)q * k, bi, sizeof(uint32_t) * (size_t)k);
        memcpy(out_d + (size_t)q * k, bd, sizeof(float) * (size_t)k);
    }
    return GOFANN_OK;
}

/* Exact filtered top-k by brute force, FP64 accumulation (the
 * filtered_topk_oracle of tests/native/quantization_smoke.py:215-238). The
 * filter is the route's DNF predicate when enabled, else the residual label
 * check plus membership of primary_label. */
int oracle_filtered_topk(const void* base, int dtype, uint32_t n_samples, uint32_t dim,
                         const void* queries, const gofann_attrs* a, const gofann_routes* r,
                         int k, uint32_t* out_ids, double* out_d)
{
    for (uint32_t route = 0; route < r->n_routes; ++route) {
        const uint32_t row = r->query_row[route];
        uint32_t bi[GOFANN_MAX_TOPK];
        double bd[GOFANN_MAX_TOPK];
        int n = 0;
        for (uint32_t s = 0; s < n_samples; ++s) {
            int ok;
            if (oracle_pred_enabled(r, route)) ok = oracle_pred_matches(r, a, route, s);
            else {
                ok = oracle_labels_match(r, a, route, s);
                if (ok && r->primary_label && r->primary_label[route] != U32MAX)
                    ok = csr_contains(a, s, r->primary_label[route]);
            }
            if (!ok) continue;
            double acc = 0.0;
            for (uint32_t dd = 0; dd < dim; ++dd) {
                double x, q;
                if (dtype == GOFANN_DTYPE_U8) {
                    x = ((const uint8_t*)base)[(size_t)s * dim + dd];
                    q = ((const uint8_t*)queries)[(size_t)row * dim + dd];
                } else if (dtype == GOFANN_DTYPE_F32) {
                    x = ((const float*)base)[(size_t)s * dim + dd];
                    q = ((const float*)queries)[(size_t)row * dim + dd];
                } else {
                    x = f16_decode(((const uint16_t*)base)[(size_t)s * dim + dd]);
                    q = ((const float*)queries)[(size_t)row * dim + dd];
                }
                acc += (x - q) * (x - q);
            }
            /* insertion into a sorted list by (dist, id) */
            int pos = n < k ? n : k;
            if (n == k && !(acc < bd[k - 1] || (acc == bd[k - 1] && s < bi[k - 1]))) continue;
            if (n < k) ++n;
            pos = n - 1;
            while (pos > 0 && (acc < bd[pos - 1] || (acc == bd[pos - 1] && s < bi[pos - 1]))) {
                bd[pos] = bd[pos - 1]; bi[pos] = bi[pos - 1]; --pos;
            }
            bd[pos] = acc; bi[pos] = s;
        }
        for (int i = 0; i < k; ++i) {
            out_ids[(size_t)route * k + i] = i < n ? bi[i] : U32MAX;
            out_d[(size_t)route * k + i] = i < n ? bd[i] : INFINITY;
        }
    }
    return GOFANN_OK;
}

/* ------------------------------------------- reference-structure probes */
/* Sequence drivers used to pin the restated heaps and hash against the
 * reference's own headers compiled in oracle/_ref (see ref_harness.cpp). */

/* Applies `n` SMMH operations: op[i] = 0 insert (key[i], payload[i]), 1
 * pop_max, 2 pop_min.  Writes the final array (first/second) and the popped
 * payloads. Returns final size. */
int oracle_seq_smmh(const int* op, const float* key, const uint32_t* payload, int n,
                    float* out_first, uint32_t* out_second, uint32_t* popped)
{
    fpair* h = (fpair*)calloc((size_t)n + 2, sizeof(fpair));
    int size = 1, np = 0;
    for (int i = 0; i < n; ++i) {
        if (op[i] == 0) {
            fpair e = {key[i], payload[i], key[i]};
            oracle_smmh_insert(h, &size, e);
        } else if (op[i] == 1 && size > 2) {
            popped[np++] = oracle_smmh_pop_max(h, &size).second;
        } else if (op[i] == 2 && size > 1) {
            popped[np++] = oracle_smmh_pop_min(h, &size).second;
        }
    }
    for (int i = 0; i < size; ++i) { out_first[i] = h[i].first; out_second[i] = h[i].second; }
    free(h);
    return size;
}

/* Bounded max-heap exactly as the traversal's result heap: keep `cap`
 * smallest by push/pop; returns the pop order (descending). */
int oracle_seq_result_heap(const float* key, const uint32_t* payload, int n, int cap,
                           float* out_first, uint32_t* out_second)
{
    rpair* b = (rpair*)calloc((size_t)cap + 2, sizeof(rpair));
    int size = 0;
    for (int i = 0; i < n; ++i) {
        rpair e = {key[i], payload[i]};
        if (size < cap) { b[size++] = e; rheap_push(b, size); }
        else if (e.first < b[0].first) {
            b[size++] = e; rheap_push(b, size); rheap_pop(b, size); --size;
        }
    }
    const int total = size;
    for (int i = 0; i < total; ++i) {
        rpair r = rheap_pop(b, total - i);
        out_first[i] = r.first; out_second[i] = r.second;
    }
    free(b);
    return total;
}

/* Inserts values into a fresh 4096-slot table; writes the table and per-add
 * outcomes (0 inserted, 1 existing, 2 full). */
void oracle_seq_hash(const uint32_t* values, int n, uint32_t* table, int32_t* outcome)
{
    for (int i = 0; i < HASH_CAP; ++i) table[i] = U32MAX;
    for (int i = 0; i < n; ++i) outcome[i] = oracle_hash_add(table, values[i]);
}

/* ------------------------------------------------- Full-GPU exact mode */
/* l2_distance_device, backend_full_gpu.cu:1106-1190: u8 as the integer
 * |x|^2 + |q|^2 - 2 x.q of dp4a (the sum of squared differences) converted
 * to float; f32 lane partials over d = l, l+32, ... (`partial += diff *
 * diff`, contracted to fma), then the shfl_down tree; f16 with an even dim
 * over half2 pairs p = l, l+32, ...: partial + (dx*dx + dy*dy), the pair term
 * contracted as fma(dx, dx, dy*dy).  Queries have the base's dtype. */
float oracle_full_l2(const void* base, int dtype, uint32_t dim, uint32_t sample, const void* queries,
                     uint32_t row)
{
    if (dtype == GOFANN_DTYPE_U8) {
        const uint8_t* b = (const uint8_t*)base + (size_t)sample * dim;
        const uint8_t* q = (const uint8_t*)queries + (size_t)row * dim;
        uint32_t acc = 0;
        for (uint32_t d = 0; d < dim; ++d) {
            const int diff = (int)b[d] - (int)q[d];
            acc += (uint32_t)(diff * diff);
        }
        return (float)acc;
    }
    float v[KW];
    for (int l = 0; l < KW; ++l) v[l] = 0.0f;
    if (dtype == GOFANN_DTYPE_F32) {
        const float* b = (const float*)base + (size_t)sample * dim;
        const float* q = (const float*)queries + (size_t)row * dim;
        for (uint32_t d = 0; d < dim; ++d) {
            const float diff = b[d] - q[d];
            v[d % KW] = fmaf(diff, diff, v[d % KW]);
        }
    } else {
        const uint16_t* b = (const uint16_t*)base + (size_t)sample * dim;
        const uint16_t* q = (const uint16_t*)queries + (size_t)row * dim;
        if ((dim & 1u) == 0) {
            for (uint32_t p = 0; p < dim / 2; ++p) {
                const float dx = f16_decode(b[2 * p]) - f16_decode(q[2 * p]);
                const float dy = f16_decode(b[2 * p + 1]) - f16_decode(q[2 * p + 1]);
                v[p % KW] = v[p % KW] + fmaf(dx, dx, dy * dy);
            }
        } else {
            for (uint32_t d = 0; d < dim; ++d) {
                const float diff = f16_decode(b[d]) - f16_decode(q[d]);
                v[d % KW] = fmaf(diff, diff, v[d % KW]);
            }
        }
    }
    return oracle_warp_sum(v);
}

/* better_result / insert_best_result, backend_full_gpu.cu:1328-1375 */
static int full_better(float ld, uint32_t li, float rd, uint32_t ri)
{
    return ld < rd || (ld == rd && li < ri);
}
static int full_insert_best(float dist, uint32_t id, int topk, float* bd, uint32_t* bi, int* size)
{
    int changed = 0;
    for (int i = 0; i < *size; ++i) {
        if (bi[i] == id) {
            if (dist >= bd[i]) return 0;
            for (int j = i; j + 1 < *size; ++j) { bd[j] = bd[j + 1]; bi[j] = bi[j + 1]; }
            --*size;
            changed = 1;
            break;
        }
    }
    if (*size == topk && !full_better(dist, id, bd[topk - 1], bi[topk - 1])) return changed;
    int pos = *size;
    if (*size < topk) ++*size; else pos = topk - 1;
    while (pos > 0 && full_better(dist, id, bd[pos - 1], bi[pos - 1])) {
        bd[pos] = bd[pos - 1];
        bi[pos] = bi[pos - 1];
        --pos;
    }
    bd[pos] = dist;
    bi[pos] = id;
    return 1;
}

/* candidate_passes_device, backend_full_gpu.cu:1015-1092, with the route's
 * filter expressed by its descriptor: the filter bit against the row mask,
 * the active range atoms, the residual labels. */
static int full_passes(const gofann_graph* g, const gofann_attrs* a, const gofann_routes* r, uint32_t route,
                       uint64_t qbit, uint32_t grow, uint32_t sample)
{
    const uint64_t mask = g->row_filter_mask ? g->row_filter_mask[grow] : ~0ull;
    if (qbit == 0 || (mask & qbit) == 0) return 0;
    const uint32_t active = count_active(r, route);
    if (active != 0 && (!a->range_values || count_matching(r, a, route, sample) != active)) return 0;
    return oracle_labels_match(r, a, route, sample);
}

/* pickup_next_unused_from_pool_block, backend_full_gpu.cu:1536-1596: the
 * unused entry of smallest distance, the smallest index among equals. */
static int full_pickup(fpair* f, int size, fpair* out)
{
    int best = -1;
    for (int i = 1; i < size; ++i) {
        if (f[i].second & POOL_USED) continue;
        if (best < 0 || f[i].first < f[best].first) best = i;
    }
    if (best < 0) return 0;
    *out = f[best];
    f[best].second |= POOL_USED;
    return 1;
}

typedef struct {
    const gofann_graph* g; const uint32_t* label_size; const gofann_attrs* a; const void* base; int dtype;
    uint32_t dim; const void* queries; const gofann_routes* r; const gofann_search_params* sp;
    uint32_t* ids; float* d; int32_t* steps; uint32_t* trace; uint32_t trace_width;
    uint32_t begin, end, stride;
} full_job;

/* One graph route of run_full_gpu_highfreq_route (backend_full_gpu.cu:
 * 1682-2043). */
static void full_search_one(const full_job* j, uint32_t route, uint32_t* hash, fpair* pool)
{
    const gofann_graph* g = j->g;
    const gofann_attrs* a = j->a;
    const gofann_routes* r = j->r;
    const gofann_search_params* sp = j->sp;
    const int QS = sp->queue_size, K = sp->result_width;
    uint32_t* oid = j->ids + (size_t)route * K;
    float* od = j->d + (size_t)route * K;
    uint32_t* tr = j->trace ? j->trace + (size_t)route * j->trace_width : NULL;
    float bd[GOFANN_MAX_TOPK];
    uint32_t bi[GOFANN_MAX_TOPK];
    int bsize = 0, steps = 0, expanded = 0, passed = 0, fh = 0;
    for (int i = 0; i < K; ++i) { oid[i] = U32MAX; od[i] = FLT_MAX; }
    if (tr) for (uint32_t i = 0; i < j->trace_width; ++i) tr[i] = U32MAX;
    if (j->steps) j->steps[route] = 0;
    const uint32_t grp = r->group_id[route];
    if (grp >= g->group_count) return;
    const uint32_t off = g->label_offset[grp];
    uint32_t gsize = j->label_size ? j->label_size[grp]
                                   : (grp + 1 < g->group_count ? g->label_offset[grp + 1] : g->total_rows) - off;
    if (off > g->total_rows || gsize > g->total_rows - off) gsize = 0;
    const uint32_t seed = r->start_local[route];
    if (gsize == 0 || seed >= gsize) return;
    const uint32_t qrow = r->query_row[route];
    const uint64_t qbit = r->filter_bits ? r->filter_bits[route] : ~0ull;
    const uint32_t seed_sample = g->row_to_sample[off + seed];
    if (seed_sample >= a->n_samples) return;
    for (int i = 0; i < HASH_CAP; ++i) hash[i] = U32MAX;
    int hs = 1;
    fpair e;
    e.first = oracle_full_l2(j->base, j->dtype, j->dim, seed_sample, j->queries, qrow);
    e.second = seed;
    e.base = e.first;
    oracle_smmh_insert(pool, &hs, e);
    oracle_hash_add(hash, seed);
    fpair now, next;
    if (!full_pickup(pool, hs, &now)) return;
    int first_step = 1;
    const int cap = sp->max_steps > 0 ? sp->max_steps : (1 << 22);
    const uint32_t deg = g->degree < GOFANN_MAX_DEGREE ? g->degree : GOFANN_MAX_DEGREE;
    uint32_t cand_local[GOFANN_MAX_DEGREE];
    float cand_d[GOFANN_MAX_DEGREE];
    for (;;) {
        if (steps >= cap) break;
        const uint32_t now_local = now.second & ~POOL_USED;
        const uint32_t now_row = off + now_local;
        const uint32_t now_sample = g->row_to_sample[now_row];
        int improved = 0;
        if (tr && (uint32_t)expanded < j->trace_width) tr[expanded] = now_local;
        ++expanded;
        if (now_sample < a->n_samples && full_passes(g, a, r, route, qbit, now_row, now_sample)) {
            ++passed;
            improved = full_insert_best(now.first, now_sample, K, bd, bi, &bsize);
        }
        ++steps;
        /* every edge tested against the table before any insertion */
        for (uint32_t ed = 0; ed < deg; ++ed) {
            cand_local[ed] = U32MAX;
            const uint32_t local = g->adjacency[(size_t)now_row * g->degree + ed];
            if (local == U32MAX || local >= gsize || oracle_hash_test(hash, local)) continue;
            const uint32_t s = g->row_to_sample[off + local];
            if (s >= a->n_samples) continue;
            cand_local[ed] = local;
            cand_d[ed] = oracle_full_l2(j->base, j->dtype, j->dim, s, j->queries, qrow);
        }
        for (uint32_t ed = 0; ed < deg; ++ed) {
            if (cand_local[ed] == U32MAX) continue;
            if (hs > 2 && hs >= QS + 1 && pool[2].first < cand_d[ed]) continue;
            fpair kp;
            kp.first = cand_d[ed];
            kp.second = cand_local[ed];
            kp.base = kp.first;
            oracle_smmh_insert(pool, &hs, kp);
            oracle_hash_add(hash, cand_local[ed]);
            if (hs >= QS + 2) oracle_smmh_pop_max(pool, &hs);
        }
        if (!full_pickup(pool, hs, &next)) break;
        if (!first_step) {
            const uint32_t next_sample = g->row_to_sample[off + (next.second & ~POOL_USED)];
            if (sp->early_stop_mode == GOFANN_EARLY_STOP_ADAPTIVE && improved) {
                fh = 0;
            } else if (bsize == K && !full_better(next.first, next_sample, bd[K - 1], bi[K - 1])) {
                ++fh;
                if (early_stop(sp->early_stop_mode, fh, sp->finish_limit, QS, expanded, passed, K)) break;
            } else {
                fh = 0;
            }
        }
        now = next;
        first_step = 0;
    }
    for (int i = 0; i < bsize; ++i) { oid[i] = bi[i]; od[i] = bd[i]; }
    if (j->steps) j->steps[route] = steps;
}

static void* full_worker(void* arg)
{
    full_job* j = (full_job*)arg;
    uint32_t* hash = (uint32_t*)malloc(HASH_CAP * sizeof(uint32_t));
    fpair* pool = (fpair*)malloc((size_t)(j->sp->queue_size + 3) * sizeof(fpair));
    for (uint32_t route = j->begin; route < j->end; route += j->stride) full_search_one(j, route, hash, pool);
    free(hash);
    free(pool);
    return NULL;
}

int oracle_exact_search(const gofann_graph* g, const uint32_t* label_size, const gofann_attrs* a,
                        const void* base, int dtype, uint32_t dim, const void* queries, const gofann_routes* r,
                        const gofann_search_params* sp, uint32_t* ids, float* d, int32_t* steps,
                        uint32_t* trace, uint32_t trace_width, int threads)
{
    if (sp->queue_size < 2 || sp->queue_size > GOFANN_MAX_QUEUE || sp->result_width < 1 ||
        sp->result_width > GOFANN_MAX_TOPK)
        return GOFANN_ERR_INVALID;
    if (threads < 1) threads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    full_job* jobs = (full_job*)malloc(sizeof(full_job) * (size_t)threads);
    for (int t = 0; t < threads; ++t) {
        full_job jb = {g, label_size, a, base, dtype, dim, queries, r, sp, ids, d, steps, trace, trace_width,
                       (uint32_t)t, r->n_routes, (uint32_t)threads};
        jobs[t] = jb;
        if (threads == 1) full_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, full_worker, &jobs[t]);
    }
    if (threads > 1)
        for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
    return GOFANN_OK;
}

/* full_gpu_lowfreq_kernel, backend_full_gpu.cu:2124-2260: every posting
 * member passing the route's filter (here its DNF predicate) is scored
 * exactly and inserted into the sorted top-k. */
int oracle_exact_posting_scan(const void* base, int dtype, uint32_t dim, const void* queries,
                              const gofann_attrs* a, const gofann_routes* r, const uint32_t* posting_ids,
                              const uint64_t* route_begin, const uint32_t* route_count, int k,
                              uint32_t* out_ids, float* out_d)
{
    if (k < 1 || k > GOFANN_MAX_SHORTLIST) return GOFANN_ERR_INVALID;
    float* bd = (float*)malloc(sizeof(float) * (size_t)k);
    uint32_t* bi = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)k);
    for (uint32_t route = 0; route < r->n_routes; ++route) {
        int size = 0;
        const uint32_t row = r->query_row[route];
        const int pred_on = oracle_pred_enabled(r, route);
        for (uint32_t i = 0; i < route_count[route]; ++i) {
            const uint32_t s = posting_ids[route_begin[route] + i];
            if (s == U32MAX || s >= a->n_samples) continue;
            if (pred_on && !oracle_pred_matches(r, a, route, s)) continue;
            full_insert_best(oracle_full_l2(base, dtype, dim, s, queries, row), s, k, bd, bi, &size);
        }
        for (int i = 0; i < k; ++i) {
            out_ids[(size_t)route * k + i] = i < size ? bi[i] : U32MAX;
            out_d[(size_t)route * k + i] = i < size ? bd[i] : FLT_MAX;
        }
    }
    free(bd);
    free(bi);
    return GOFANN_OK;
}

/* The entry full_pickup() takes from a frontier of `size` entries (index 0
 * unused; vals carry the used bit), or -1; nothing is modified. */
int oracle_full_pickup_index(const float* keys, const uint32_t* vals, int size)
{
    fpair* f = (fpair*)calloc((size_t)(size > 1 ? size : 1), sizeof(fpair));
    for (int i = 0; i < size; ++i) { f[i].first = keys[i]; f[i].second = vals[i]; f[i].base = keys[i]; }
    fpair out;
    int idx = -1;
    if (full_pickup(f, size, &out)) idx = (int)(out.second & ~POOL_USED);
    free(f);
    return idx;
}
